"""Bandwidth contention generator (a TCP flood to a sink) used to emulate a slow link.

    python -m resihp_megatron_b200.inject.contention --host H --port P --seconds S [--serve]
(Reference: ``resihp/inject/contention.py``.)
"""

from __future__ import annotations

import argparse
import socket
import threading
import time


def sink(port: int, seconds: float, host: str = "0.0.0.0") -> int:
    """Accept connections and discard everything for ``seconds``; returns bytes received."""
    srv = socket.create_server((host, port))
    srv.settimeout(0.2)
    total = [0]
    deadline = time.monotonic() + seconds

    def drain(c: socket.socket) -> None:
        c.settimeout(0.2)
        while time.monotonic() < deadline:
            try:
                b = c.recv(1 << 20)
            except socket.timeout:
                continue
            except OSError:
                break
            if not b:
                break
            total[0] += len(b)
        c.close()

    while time.monotonic() < deadline:
        try:
            c, _ = srv.accept()
        except socket.timeout:
            continue
        threading.Thread(target=drain, args=(c,), daemon=True).start()
    srv.close()
    return total[0]


def flood(host: str, port: int, seconds: float, streams: int = 4, chunk: int = 1 << 20) -> int:
    """Push data to ``host:port`` on ``streams`` connections for ``seconds``; returns bytes sent."""
    buf = b"\0" * chunk
    sent = [0] * streams
    deadline = time.monotonic() + seconds

    def push(i: int) -> None:
        try:
            s = socket.create_connection((host, port), timeout=5)
        except OSError:
            return
        with s:
            while time.monotonic() < deadline:
                try:
                    s.sendall(buf)
                    sent[i] += len(buf)
                except OSError:
                    return

    ts = [threading.Thread(target=push, args=(i,), daemon=True) for i in range(streams)]
    for t in ts:
        t.start()
    for t in ts:
        t.join(seconds + 5)
    return sum(sent)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="resihp-contention")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=29700)
    ap.add_argument("--seconds", type=float, default=60.0)
    ap.add_argument("--streams", type=int, default=4)
    ap.add_argument("--serve", action="store_true", help="run the sink instead of the flood")
    a = ap.parse_args(argv)
    n = sink(a.port, a.seconds) if a.serve else flood(a.host, a.port, a.seconds, a.streams)
    print(n)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
