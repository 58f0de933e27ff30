"""Control-plane messaging: one JSON object per line over a TCP stream.

The control plane never shares a socket or a thread with the data plane (NCCL / peer
kernels), so it keeps working while a collective is wedged.  Each ``Connection`` owns one
reader thread that hands decoded messages to a callback; writes are serialised by a lock.
Public names follow the reference (``resihp/utils/rpc.py:23-164``): ``Connection``,
``Server``, ``connect``, ``parse_addr``, ``fmt_addr``.
"""

from __future__ import annotations

import json
import socket
import threading
import time
from typing import Callable

from .log import get_logger

log = get_logger(__name__)

MessageHandler = Callable[["Connection", dict], None]
CloseHandler = Callable[["Connection"], None]


class Connection:
    """Bidirectional message channel; ``on_message`` runs on the reader thread."""

    def __init__(self, sock: socket.socket, on_message: MessageHandler,
                 on_close: CloseHandler | None = None, name: str = ""):
        self.sock = sock
        try:
            sock.setsockopt(socket.IPPROTO_TCP, socket.TCP_NODELAY, 1)
        except OSError:
            pass
        self.meta: dict = {}
        self._handler = on_message
        self._close_cb = on_close
        self._send_lock = threading.Lock()
        self._state_lock = threading.Lock()
        self._closed = threading.Event()
        self._thread = threading.Thread(target=self._pump, name=f"rpc-{name}", daemon=True)
        self._thread.start()

    @property
    def closed(self) -> bool:
        return self._closed.is_set()

    def send(self, msg: dict) -> bool:
        line = json.dumps(msg, separators=(",", ":")).encode() + b"\n"
        with self._send_lock:
            if self._closed.is_set():
                return False
            try:
                self.sock.sendall(line)
                return True
            except OSError:
                failed = True
        if failed:
            self.close()
        return False

    def _pump(self) -> None:
        buf = b""
        try:
            while True:
                chunk = self.sock.recv(65536)
                if not chunk:
                    break
                buf += chunk
                while True:
                    nl = buf.find(b"\n")
                    if nl < 0:
                        break
                    line, buf = buf[:nl], buf[nl + 1:]
                    if not line.strip():
                        continue
                    try:
                        msg = json.loads(line)
                    except ValueError:
                        log.warning("dropping malformed control message")
                        continue
                    try:
                        self._handler(self, msg)
                    except Exception:  # noqa: BLE001 - a faulty handler must not kill the channel
                        log.exception("handler raised on %s", msg.get("type"))
        except OSError:
            pass
        finally:
            self.close()

    def close(self) -> None:
        with self._state_lock:
            if self._closed.is_set():
                return
            self._closed.set()
        for op in (lambda: self.sock.shutdown(socket.SHUT_RDWR), self.sock.close):
            try:
                op()
            except OSError:
                pass
        if self._close_cb is not None:
            try:
                self._close_cb(self)
            except Exception:  # noqa: BLE001
                log.exception("close callback raised")


class Server:
    """Accepts connections and wraps each one in a ``Connection``."""

    def __init__(self, host: str, port: int, on_message: MessageHandler,
                 on_connect: Callable[[Connection], None] | None = None,
                 on_close: CloseHandler | None = None):
        self._on_message = on_message
        self._on_connect = on_connect
        self._on_close = on_close
        self._listener = socket.create_server((host, port), backlog=1024)
        self.address: tuple[str, int] = self._listener.getsockname()[:2]
        self.connections: set[Connection] = set()
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._accept, name="rpc-accept", daemon=True)
        self._thread.start()

    def _accept(self) -> None:
        while not self._stop.is_set():
            try:
                s, _ = self._listener.accept()
            except OSError:
                return
            if self._stop.is_set():  # accepted while stopping: refuse
                s.close()
                return
            c = Connection(s, self._on_message, self._forget)
            with self._lock:
                self.connections.add(c)
            if self._on_connect is not None:
                self._on_connect(c)

    def _forget(self, c: Connection) -> None:
        with self._lock:
            self.connections.discard(c)
        if self._on_close is not None:
            self._on_close(c)

    def stop(self) -> None:
        self._stop.set()
        # shutdown() first: a bare close() leaves a listener that another thread is blocked in
        # accept() on still accepting connections on Linux
        for op in (lambda: self._listener.shutdown(socket.SHUT_RDWR), self._listener.close):
            try:
                op()
            except OSError:
                pass
        with self._lock:
            live = list(self.connections)
        for c in live:
            c.close()


def connect(addr: tuple[str, int], on_message: MessageHandler, on_close: CloseHandler | None = None,
            timeout: float = 10.0, retry_interval: float = 0.05, name: str = "") -> Connection:
    """Dial ``addr``, retrying until ``timeout``; raises ``TimeoutError`` when it never answers."""
    give_up = time.monotonic() + timeout
    err: Exception | None = None
    while True:
        try:
            s = socket.create_connection(addr, timeout=min(2.0, max(timeout, 0.05)))
            s.settimeout(None)
            return Connection(s, on_message, on_close, name=name)
        except OSError as e:
            err = e
        if time.monotonic() >= give_up:
            raise TimeoutError(f"could not connect to {addr}: {err}")
        time.sleep(retry_interval)


def parse_addr(s: str) -> tuple[str, int]:
    host, _, port = s.rpartition(":")
    return host, int(port)


def fmt_addr(addr) -> str:
    return f"{addr[0]}:{addr[1]}"
