"""T2: persistent checkpoints stored as logical slices, loadable by any later plan.

On-disk format (kept identical to the reference, ``resihp/state/checkpoint.py:23-135``):
``<root>/iter_<it:08d>/<owner>.pt`` written as ``.<owner>.pt.tmp`` then atomically renamed;
content ``torch.save({"slices": [(SliceMeta.to_json(), {kind: cpu tensor})], "extra": {...}})``;
``<owner>.done`` holds the JSON list of the owner's slice metas (written last = the commit
marker).  A ``SliceMeta`` is ``{"key", "global_shape", "dim" (null = replicated), "interval"}``;
replicated tensors use the interval ``[0, 1]``.  Loading assembles any requested interval from
whichever saved slices overlap it (reshard on load for arbitrary TP / PP / DP changes).
Saving runs on a background thread after a synchronous device-to-host copy.
"""

from __future__ import annotations

import json
import os
import threading
from dataclasses import dataclass
from pathlib import Path

import torch

from ..utils.intervals import intersect


@dataclass(frozen=True)
class SliceMeta:
    key: str
    global_shape: tuple[int, ...]
    dim: int | None
    interval: tuple[int, int]

    def to_json(self) -> dict:
        return {"key": self.key, "global_shape": list(self.global_shape), "dim": self.dim,
                "interval": list(self.interval)}

    @staticmethod
    def from_json(d: dict) -> "SliceMeta":
        return SliceMeta(d["key"], tuple(d["global_shape"]), d["dim"], tuple(d["interval"]))


class SliceCheckpointer:
    def __init__(self, directory: str | os.PathLike):
        self.root = Path(directory)
        self._thread: threading.Thread | None = None

    def _dir(self, iteration: int) -> Path:
        return self.root / f"iter_{iteration:08d}"

    def save(self, iteration: int, owner: str, slices: list[tuple[SliceMeta, dict[str, torch.Tensor]]],
             extra: dict | None = None, blocking: bool = False) -> None:
        self.wait()
        host = [(m, {k: v.detach().to("cpu", copy=True) for k, v in t.items()}) for m, t in slices]

        def write() -> None:
            d = self._dir(iteration)
            d.mkdir(parents=True, exist_ok=True)
            tmp = d / f".{owner}.pt.tmp"
            torch.save({"slices": [(m.to_json(), t) for m, t in host], "extra": extra or {}}, tmp)
            os.replace(tmp, d / f"{owner}.pt")
            (d / f"{owner}.done").write_text(json.dumps([m.to_json() for m, _ in host]))

        if blocking:
            write()
        else:
            self._thread = threading.Thread(target=write, name="ckpt-save", daemon=True)
            self._thread.start()

    def wait(self) -> None:
        if self._thread is not None:
            self._thread.join()
            self._thread = None

    def _index(self, iteration: int) -> list[tuple[str, SliceMeta]]:
        out = []
        for done in sorted(self._dir(iteration).glob("*.done")):
            owner = done.name[: -len(".done")]
            out.extend((owner, SliceMeta.from_json(m)) for m in json.loads(done.read_text()))
        return out

    def complete(self, iteration: int, required: dict[str, tuple[tuple[int, ...], int | None]]) -> bool:
        idx = self._index(iteration)
        for key, (shape, dim) in required.items():
            n = shape[dim] if dim is not None else 1
            reach = 0
            for a, b in sorted(m.interval for _, m in idx if m.key == key):
                if a > reach:
                    return False
                reach = max(reach, b)
            if reach < n:
                return False
        return True

    def latest_complete(self, required: dict[str, tuple[tuple[int, ...], int | None]]) -> int | None:
        if not self.root.exists():
            return None
        its = sorted((int(p.name[5:]) for p in self.root.glob("iter_*")), reverse=True)
        for it in its:
            if self.complete(it, required):
                return it
        return None

    def read_extra(self, iteration: int, owner: str) -> dict:
        return torch.load(self._dir(iteration) / f"{owner}.pt", weights_only=False).get("extra", {})

    def load(self, iteration: int, wanted: list[SliceMeta], kinds: tuple[str, ...]) -> dict[str, dict[str, torch.Tensor]]:
        idx = self._index(iteration)
        files: dict[str, list] = {}
        out: dict[str, dict[str, torch.Tensor]] = {}
        for want in wanted:
            dim = want.dim
            shape = list(want.global_shape)
            if dim is not None:
                shape[dim] = want.interval[1] - want.interval[0]
            got: dict[str, torch.Tensor | None] = dict.fromkeys(kinds)
            covered = 0
            for owner, meta in idx:
                if meta.key != want.key:
                    continue
                o = intersect(meta.interval, want.interval) if dim is not None else (0, 1)
                if o is None:
                    continue
                if owner not in files:
                    files[owner] = torch.load(self._dir(iteration) / f"{owner}.pt", weights_only=False)["slices"]
                tensors = next(t for m, t in files[owner] if SliceMeta.from_json(m) == meta)
                for k in kinds:
                    if got[k] is None:
                        got[k] = torch.empty(shape, dtype=tensors[k].dtype)
                    if dim is None:
                        got[k].copy_(tensors[k])
                    else:
                        got[k].narrow(dim, o[0] - want.interval[0], o[1] - o[0]).copy_(
                            tensors[k].narrow(dim, o[0] - meta.interval[0], o[1] - o[0]))
                covered += (o[1] - o[0]) if dim is not None else 1
                if dim is None:
                    break
            if covered < ((want.interval[1] - want.interval[0]) if dim is not None else 1):
                raise KeyError(f"checkpoint {iteration} does not cover {want}")
            out[want.key] = got
        return out
