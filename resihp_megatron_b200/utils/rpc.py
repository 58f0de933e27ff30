"""Control-plane messaging: newline-delimited JSON objects over TCP.

The control plane never shares a socket or a thread with the data plane (NCCL, peer-memory
kernels), so it keeps answering while a collective is wedged.  Every ``Connection`` runs one
reader thread that decodes lines and hands each message to its callback; writers share a lock.
A connection closes once, from whichever side notices first, and then runs its close callback.
The wire format (one compact JSON object per ``\\n``-terminated line) and the public names
``Connection``, ``Server``, ``connect``, ``parse_addr`` and ``fmt_addr`` are the reference's
(``resihp/utils/rpc.py:23-164``), so processes of either framework can talk to each other.
"""

from __future__ import annotations

import contextlib
import json
import socket
import threading
import time
from typing import Callable

from .log import get_logger

log = get_logger(__name__)

MessageHandler = Callable[["Connection", dict], None]
CloseHandler = Callable[["Connection"], None]


def _encode(message: dict) -> bytes:
    return (json.dumps(message, separators=(",", ":")) + "\n").encode()


class Connection:
    """One bidirectional message channel; ``on_message`` runs on its reader thread."""

    def __init__(self, sock: socket.socket, on_message: MessageHandler,
                 on_close: CloseHandler | None = None, name: str = ""):
        with contextlib.suppress(OSError):  # small control messages: no Nagle delay
            sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        self.sock, self.meta = sock, {}
        self._on_message, self._on_close = on_message, on_close
        self._write = threading.Lock()
        self._closing = threading.Lock()
        self._done = threading.Event()
        threading.Thread(target=self._read_loop, name=f"rpc-{name}", daemon=True).start()

    @property
    def closed(self) -> bool:
        return self._done.is_set()

    def send(self, msg: dict) -> bool:
        """Write one message; False (and the channel closed) when the peer is gone."""
        data = _encode(msg)
        delivered = False
        with self._write:
            if not self._done.is_set():
                with contextlib.suppress(OSError):
                    self.sock.sendall(data)
                    delivered = True
                broken = not delivered
            else:
                broken = False
        if broken:
            self.close()
        return delivered

    def _deliver(self, raw: bytes) -> None:
        if not raw.strip():
            return
        try:
            message = json.loads(raw)
        except ValueError:
            log.warning("dropping malformed control message")
            return
        try:
            self._on_message(self, message)
        except Exception:  # noqa: BLE001 -- a faulty handler must not take the channel down
            log.exception("handler raised on %s", message.get("type"))

    def _read_loop(self) -> None:
        with contextlib.suppress(OSError, ValueError), self.sock.makefile("rb") as stream:
            for raw in stream:
                self._deliver(raw)
        self.close()

    def close(self) -> None:
        with self._closing:
            first = not self._done.is_set()
            self._done.set()
        if not first:
            return
        _teardown(self.sock)
        callback = self._on_close
        if callback is None:
            return
        with contextlib.suppress(Exception):
            callback(self)


def _teardown(sock: socket.socket) -> None:
    """Shut a socket down in both directions, then release it (errors ignored)."""
    for step in (lambda: sock.shutdown(socket.SHUT_RDWR), sock.close):
        with contextlib.suppress(OSError):
            step()


class Server:
    """Listens on ``(host, port)`` (port 0: any) and wraps each accepted socket."""

    def __init__(self, host: str, port: int, on_message: MessageHandler,
                 on_connect: Callable[[Connection], None] | None = None,
                 on_close: CloseHandler | None = None):
        self._on_message, self._on_connect, self._on_close = on_message, on_connect, on_close
        self._sock = socket.create_server((host, port), backlog=1024)
        self.address: tuple[str, int] = tuple(self._sock.getsockname()[:2])
        self.connections: set[Connection] = set()
        self._mu = threading.Lock()
        self._halt = threading.Event()
        threading.Thread(target=self._serve, name="rpc-accept", daemon=True).start()

    def _next_socket(self) -> socket.socket | None:
        with contextlib.suppress(OSError):
            sock, _peer = self._sock.accept()
            if not self._halt.is_set():
                return sock
            sock.close()
        return None

    def _serve(self) -> None:
        while (sock := self._next_socket()) is not None:
            conn = Connection(sock, self._on_message, self._dropped)
            with self._mu:
                self.connections.add(conn)
            hook = self._on_connect
            if hook:
                hook(conn)

    def _dropped(self, conn: Connection) -> None:
        with self._mu:
            self.connections.discard(conn)
        hook = self._on_close
        if hook:
            hook(conn)

    def stop(self) -> None:
        self._halt.set()
        # the listener is shut down before it is closed: on Linux a bare close() leaves a thread
        # blocked in accept() still accepting
        _teardown(self._sock)
        with self._mu:
            open_conns = list(self.connections)
        for conn in open_conns:
            conn.close()


def connect(addr: tuple[str, int], on_message: MessageHandler, on_close: CloseHandler | None = None,
            timeout: float = 10.0, retry_interval: float = 0.05, name: str = "") -> Connection:
    """Dial ``addr`` until it answers or ``timeout`` passes (then ``TimeoutError``)."""
    give_up_at = time.monotonic() + timeout
    dial_timeout = min(2.0, max(timeout, 0.05))
    attempts: list[OSError] = []
    while not attempts or time.monotonic() < give_up_at:
        if attempts:
            time.sleep(retry_interval)
        with contextlib.suppress(OSError):
            sock = socket.create_connection(addr, timeout=dial_timeout)
            sock.settimeout(None)
            return Connection(sock, on_message, on_close, name=name)
        attempts.append(OSError(f"no answer from {addr}"))
    raise TimeoutError(f"could not connect to {addr} after {len(attempts)} attempts")


def parse_addr(s: str) -> tuple[str, int]:
    """``"host:port"`` -> ``(host, port)`` (the last colon splits, so IPv6 hosts work)."""
    cut = s.rindex(":")
    return s[:cut], int(s[cut + 1:])


def fmt_addr(addr) -> str:
    host, port = addr[0], addr[1]
    return f"{host}:{port}"
