"""Multi-process gloo helpers for tests on localhost (127.0.0.1)."""

from __future__ import annotations

import multiprocessing as mp
import os
import queue
import socket
import sys
import time
import traceback
from typing import Any, Callable


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(fn: Callable, rank: int, world: int, port: int, q, args: tuple) -> None:
    os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo0" if sys.platform == "darwin" else "lo")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import io

    import torch

    torch.set_num_threads(1)
    try:
        buf = io.BytesIO()
        torch.save(fn(rank, world, port, *args), buf)  # bytes, not shared-memory tensors
        q.put((rank, True, buf.getvalue()))
    except BaseException as e:  # noqa: BLE001 - report every failure to the test process
        q.put((rank, False, f"{type(e).__name__}: {e}\n{traceback.format_exc()}"))


def spawn(fn: Callable, world: int, *args: Any, timeout: float = 120.0,
          expect_dead: set[int] | None = None) -> dict[int, Any]:
    """Run ``fn(rank, world, port, *args)`` in ``world`` processes and return ``{rank: result}``;
    ranks in ``expect_dead`` may exit without reporting (killed on purpose)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(fn, r, world, port, q, args), daemon=True) for r in range(world)]
    for p in procs:
        p.start()
    dead = expect_dead or set()
    ok: dict[int, Any] = {}
    bad: dict[int, str] = {}
    deadline = time.monotonic() + timeout
    while len(ok) + len(bad) < world - len(dead) and time.monotonic() < deadline:
        try:
            r, success, payload = q.get(timeout=0.5)
        except queue.Empty:
            continue
        if success:
            import io

            import torch

            ok[r] = torch.load(io.BytesIO(payload), weights_only=False)
        else:
            bad[r] = payload
    for p in procs:
        p.join(timeout=2)
        if p.is_alive():
            p.kill()
    if bad:
        raise AssertionError("worker failures:\n" + "\n".join(f"[rank {r}] {e}" for r, e in sorted(bad.items())))
    missing = set(range(world)) - set(ok) - dead
    if missing:
        raise AssertionError(f"ranks {sorted(missing)} did not report within {timeout}s")
    return ok
