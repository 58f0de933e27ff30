"""T2: persistent checkpoints stored as logical slices, loadable into any later plan.

On-disk format -- kept identical to the reference's (``resihp/state/checkpoint.py:23-135``) so
checkpoints move between the two frameworks:

* ``<root>/iter_<it:08d>/<owner>.pt``, written as ``.<owner>.pt.tmp`` and renamed atomically,
  holding ``torch.save({"slices": [(SliceMeta.to_json(), {kind: cpu tensor})], "extra": {...}})``;
* ``<owner>.done``: the JSON list of that owner's slice metas, written last (the commit marker);
* a ``SliceMeta`` is ``{"key", "global_shape", "dim" (null: replicated), "interval"}``, and a
  replicated tensor uses the interval ``[0, 1]``.

Loading assembles any requested interval from whichever saved slices overlap it, so a
checkpoint reshards on load for arbitrary TP / PP / DP changes.  Saving copies to host memory
synchronously and writes on a background thread.
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
        return dict(key=self.key, global_shape=list(self.global_shape), dim=self.dim, interval=list(self.interval))

    @classmethod
    def from_json(cls, d: dict) -> "SliceMeta":
        return cls(d["key"], tuple(d["global_shape"]), d["dim"], tuple(d["interval"]))

    @property
    def length(self) -> int:
        return 1 if self.dim is None else self.interval[1] - self.interval[0]

    def local_shape(self) -> list[int]:
        shape = list(self.global_shape)
        if self.dim is not None:
            shape[self.dim] = self.length
        return shape


def _covers(intervals, extent: int) -> bool:
    """Whether the union of ``intervals`` contains ``[0, extent)``."""
    reach = 0
    for lo, hi in sorted(intervals):
        if lo > reach:
            break
        reach = max(reach, hi)
    return reach >= extent


class _Iteration:
    """The committed slices of one checkpoint iteration, with lazily loaded owner files."""

    def __init__(self, folder: Path):
        self.folder = folder
        self.metas: list[tuple[str, SliceMeta]] = []
        for marker in sorted(folder.glob("*.done")):
            owner = marker.name.removesuffix(".done")
            self.metas += [(owner, SliceMeta.from_json(m)) for m in json.loads(marker.read_text())]
        self._files: dict[str, dict] = {}

    def of_key(self, key: str) -> list[tuple[str, SliceMeta]]:
        return [(owner, m) for owner, m in self.metas if m.key == key]

    def tensors(self, owner: str, meta: SliceMeta) -> dict[str, torch.Tensor]:
        if owner not in self._files:
            saved = torch.load(self.folder / f"{owner}.pt", weights_only=False)["slices"]
            self._files[owner] = {SliceMeta.from_json(m): t for m, t in saved}
        return self._files[owner][meta]


class SliceCheckpointer:
    def __init__(self, directory: str | os.PathLike):
        self.root = Path(directory)
        self._writer: threading.Thread | None = None

    def _dir(self, iteration: int) -> Path:
        return self.root / f"iter_{iteration:08d}"

    def save(self, iteration: int, owner: str, slices: list[tuple[SliceMeta, dict[str, torch.Tensor]]],
             extra: dict | None = None, blocking: bool = False) -> None:
        """Write ``owner``'s slices of ``iteration`` (device tensors are copied to host first)."""
        self.wait()
        on_host = [(meta, {kind: t.detach().to("cpu", copy=True) for kind, t in per_kind.items()})
                   for meta, per_kind in slices]
        folder = self._dir(iteration)

        def persist() -> None:
            folder.mkdir(parents=True, exist_ok=True)
            partial = folder / f".{owner}.pt.tmp"
            torch.save({"slices": [(m.to_json(), t) for m, t in on_host], "extra": dict(extra or {})}, partial)
            os.replace(partial, folder / f"{owner}.pt")
            (folder / f"{owner}.done").write_text(json.dumps([m.to_json() for m, _ in on_host]))

        if blocking:
            persist()
        else:
            self._writer = threading.Thread(target=persist, name="ckpt-save", daemon=True)
            self._writer.start()

    def wait(self) -> None:
        writer, self._writer = self._writer, None
        if writer is not None:
            writer.join()

    def complete(self, iteration: int, required: dict[str, tuple[tuple[int, ...], int | None]]) -> bool:
        """Every required key fully covered by committed slices of ``iteration``."""
        found = _Iteration(self._dir(iteration))
        for key, (shape, dim) in required.items():
            extent = 1 if dim is None else shape[dim]
            if not _covers([m.interval for _, m in found.of_key(key)], extent):
                return False
        return True

    def latest_complete(self, required: dict[str, tuple[tuple[int, ...], int | None]]) -> int | None:
        if not self.root.is_dir():
            return None
        iterations = sorted((int(p.name.removeprefix("iter_")) for p in self.root.glob("iter_*")), reverse=True)
        return next((it for it in iterations if self.complete(it, required)), None)

    def read_extra(self, iteration: int, owner: str) -> dict:
        return torch.load(self._dir(iteration) / f"{owner}.pt", weights_only=False).get("extra", {})

    def load(self, iteration: int, wanted: list[SliceMeta], kinds: tuple[str, ...]) -> dict[str, dict[str, torch.Tensor]]:
        """Assemble every wanted slice from the saved slices that overlap it."""
        found = _Iteration(self._dir(iteration))
        assembled: dict[str, dict[str, torch.Tensor]] = {}
        for want in wanted:
            parts: dict[str, torch.Tensor] = {}
            filled = 0
            for owner, meta in found.of_key(want.key):
                overlap = (0, 1) if want.dim is None else intersect(meta.interval, want.interval)
                if overlap is None:
                    continue
                saved = found.tensors(owner, meta)
                for kind in kinds:
                    target = parts.setdefault(kind, torch.empty(want.local_shape(), dtype=saved[kind].dtype))
                    if want.dim is None:
                        target.copy_(saved[kind])
                        continue
                    width = overlap[1] - overlap[0]
                    target.narrow(want.dim, overlap[0] - want.interval[0], width).copy_(
                        saved[kind].narrow(want.dim, overlap[0] - meta.interval[0], width))
                filled += overlap[1] - overlap[0] if want.dim is not None else 1
                if want.dim is None:
                    break  # one copy of a replicated tensor is enough
            if filled < want.length:
                raise KeyError(f"checkpoint {iteration} does not cover {want}")
            assembled[want.key] = {kind: parts.get(kind) for kind in kinds}
        return assembled
