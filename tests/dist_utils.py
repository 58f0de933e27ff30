"""Runs a function in several spawned processes that talk over gloo on 127.0.0.1."""

from __future__ import annotations

import io
import multiprocessing as mp
import os
import queue
import socket
import sys
import time
import traceback
from typing import Any, Callable


def free_port() -> int:
    """A TCP port on 127.0.0.1 that was free a moment ago."""
    probe = socket.socket()
    try:
        probe.bind(("127.0.0.1", 0))
        return probe.getsockname()[1]
    finally:
        probe.close()


def _child(fn: Callable, rank: int, world: int, port: int, results, args: tuple) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    os.environ.setdefault("GLOO_SOCKET_IFNAME", "lo0" if sys.platform == "darwin" else "lo")
    import torch

    torch.set_num_threads(1)
    try:
        value = fn(rank, world, port, *args)
    except BaseException as err:  # noqa: BLE001 -- every failure goes back to the test
        results.put((rank, "error", f"{type(err).__name__}: {err}\n{traceback.format_exc()}"))
        return
    packed = io.BytesIO()
    torch.save(value, packed)  # plain bytes: no shared-memory tensors cross the queue
    results.put((rank, "ok", packed.getvalue()))


def spawn(fn: Callable, world: int, *args: Any, timeout: float = 120.0,
          expect_dead: set[int] | None = None) -> dict[int, Any]:
    """``fn(rank, world, port, *args)`` in ``world`` processes; returns ``{rank: result}``.
    Ranks in ``expect_dead`` may exit without a result (killed on purpose)."""
    import torch

    ctx = mp.get_context("spawn")
    results = ctx.Queue()
    port = free_port()
    children = [ctx.Process(target=_child, args=(fn, r, world, port, results, args), daemon=True)
                for r in range(world)]
    for child in children:
        child.start()
    silent = set(expect_dead or ())
    values: dict[int, Any] = {}
    errors: dict[int, str] = {}
    give_up = time.monotonic() + timeout
    while len(values) + len(errors) < world - len(silent) and time.monotonic() < give_up:
        try:
            rank, status, payload = results.get(timeout=0.5)
        except queue.Empty:
            continue
        if status == "ok":
            values[rank] = torch.load(io.BytesIO(payload), weights_only=False)
        else:
            errors[rank] = payload
    for child in children:
        child.join(timeout=2)
        if child.is_alive():
            child.kill()
    if errors:
        raise AssertionError("worker failures:\n" + "\n".join(f"[rank {r}] {e}" for r, e in sorted(errors.items())))
    unheard = sorted(set(range(world)) - set(values) - silent)
    if unheard:
        raise AssertionError(f"ranks {unheard} did not report within {timeout}s")
    return values
