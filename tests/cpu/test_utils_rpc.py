"""Control-plane transport and canonical JSON."""

import dataclasses
import threading
from enum import Enum

import pytest

from resihp_megatron_b200.utils import serialization as ser
from resihp_megatron_b200.utils.rpc import Server, connect, fmt_addr, parse_addr


def test_messages_round_trip_in_order_and_close_is_reported_once():
    got, closed = [], []
    done = threading.Event()

    def on_msg(conn, m):
        got.append(m)
        conn.send({"type": "ACK", "n": m["n"]})
        if m["n"] == 99:
            done.set()

    srv = Server("127.0.0.1", 0, on_msg, on_close=lambda c: closed.append(c))
    acks = []
    client = connect(srv.address, lambda c, m: acks.append(m["n"]), timeout=5)
    for n in range(100):
        assert client.send({"type": "PING", "n": n, "payload": "x" * (n * 50)})
    assert done.wait(5)
    assert [m["n"] for m in got] == list(range(100))
    client.close()
    client.close()
    assert client.closed and not client.send({"type": "late"})
    for _ in range(100):
        if closed:
            break
        threading.Event().wait(0.02)
    assert len(closed) == 1
    srv.stop()


def test_connect_times_out_and_addresses_parse():
    srv = Server("127.0.0.1", 0, lambda c, m: None)
    addr = srv.address
    srv.stop()
    with pytest.raises(TimeoutError):
        connect(addr, lambda c, m: None, timeout=0.2)
    assert parse_addr(fmt_addr(("::1", 80))) == ("::1", 80)


class Color(Enum):
    RED = "red"


@dataclasses.dataclass
class Rec:
    b: tuple
    a: set


def test_canonical_json_is_order_independent_and_tuplify_restores_tuples():
    one = ser.dumps({"z": Rec((1, 2), {3, 1}), "c": Color.RED})
    two = ser.dumps({"c": Color.RED, "z": Rec((1, 2), {1, 3})})
    assert one == two == '{"c":"red","z":{"a":[1,3],"b":[1,2]}}'
    assert ser.tuplify(ser.loads('{"k": [[1, 2], {"x": [3]}]}')) == {"k": ((1, 2), {"x": (3,)})}
