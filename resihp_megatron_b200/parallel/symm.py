"""Per-generation symmetric peer memory on one NVLink/NVSwitch node.

Each rank allocates one device region holding a signal pad and named segments at identical
offsets, shares it, and maps every peer's region; kernels then read and write peers' segments
directly over NVLink.  Two ways to share a region: ``"vmm"`` (the default where the driver offers
it) -- a cuMem allocation exported as a POSIX file descriptor, which each peer receives over a
Unix socket (``SCM_RIGHTS``) and maps into its own reserved range; the imported handle keeps the
physical memory alive, so a departed peer's region stays mapped for the survivors until they drop
it -- or ``"ipc"``: ``cudaMalloc`` plus a CUDA IPC handle.  A reconfiguration tears the heap down (``close``) and
builds the next generation's heap over the new world -- the counterpart of rebuilding NCCL
communicators (reference: ``resihp/comm/comm_manager.py:138-251``).

``AbortWord`` is pinned host memory mapped into the device: the control plane raises it from
the host (``ResilientCommManager.add_abort_hook``) while a kernel runs, and every bounded wait
in the peer kernels polls it, so survivors leave an in-flight fused kernel without waiting for a
timeout.  ``barrier`` is a bounded cross-GPU barrier on the signal pad; its outcome is read with
``check`` (which synchronises) and raised as ``PeerTimeout`` / ``PeerAborted``.
"""

from __future__ import annotations

import json
import os
import socket
import threading
import time
import uuid
from dataclasses import dataclass
from typing import Callable

import torch

from ..ops._build import ext

ALIGN = 256
_DTYPES = {torch.float32: "float32", torch.bfloat16: "bfloat16", torch.int32: "int32", torch.int64: "int64",
           torch.uint8: "uint8"}


class PeerTimeout(RuntimeError):
    pass


class PeerAborted(RuntimeError):
    pass


class AbortWord:
    """One host-mapped int per device context; ``set()`` is safe from any host thread."""

    def __init__(self):
        self.host, self.dev = ext().host_words_alloc(4)

    def set(self, value: int = 1) -> None:
        ext().host_word_set(self.host, 0, value)

    def clear(self) -> None:
        ext().host_word_set(self.host, 0, 0)

    @property
    def raised(self) -> bool:
        return ext().host_word_get(self.host, 0) != 0

    def close(self) -> None:
        if self.host:
            ext().host_words_free(self.host)
            self.host = self.dev = 0


@dataclass
class Segment:
    offset: int
    numel: int
    dtype: torch.dtype

    @property
    def nbytes(self) -> int:
        return self.numel * torch.empty(0, dtype=self.dtype).element_size()


SIGNAL_SLOT_BYTES = 128  # one 64-bit word per writer rank, each on its own 128-byte line (symm.cu)


def layout(segments: dict[str, tuple[int, torch.dtype]], world: int) -> tuple[dict[str, Segment], int, int]:
    """Offsets of the signal pad and of every segment; returns (segments, pad bytes, total)."""
    pad = (world * SIGNAL_SLOT_BYTES + ALIGN - 1) // ALIGN * ALIGN
    off = pad
    out = {}
    for name, (numel, dtype) in segments.items():
        seg = Segment(off, numel, dtype)
        out[name] = seg
        off += (seg.nbytes + ALIGN - 1) // ALIGN * ALIGN
    return out, pad, off


def check_layout(segs: dict[str, Segment], pad: int, total: int, world: int) -> None:
    """Invariants every rank's kernels rely on: the signal pad holds one slot per rank, every
    segment starts on an ``ALIGN`` boundary after the pad, segments do not overlap and fit."""
    if pad < world * SIGNAL_SLOT_BYTES or pad % ALIGN:
        raise AssertionError(f"signal pad of {pad} bytes for {world} ranks")
    spans = sorted((seg.offset, seg.offset + seg.nbytes, name) for name, seg in segs.items())
    end = pad
    for lo, hi, name in spans:
        if lo % ALIGN or lo < end:
            raise AssertionError(f"segment {name} at {lo} overlaps or is misaligned")
        end = hi
    if end > total:
        raise AssertionError(f"segments end at {end} beyond the heap's {total} bytes")


class _FdServer:
    """Hands this rank's region descriptor to ``peers`` connecting processes over an
    abstract-namespace Unix socket (``SCM_RIGHTS``), then stops."""

    def __init__(self, fd: int, peers: int, timeout_s: float = 60.0):
        self.fd, self.peers = fd, peers
        self.name = f"resihp-symm-{os.getpid()}-{uuid.uuid4().hex}"
        self.sock = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
        self.sock.bind("\0" + self.name)
        self.sock.listen(max(1, peers))
        self.sock.settimeout(timeout_s)
        self.error: BaseException | None = None
        self.thread = threading.Thread(target=self._serve, name="symm-fd-server", daemon=True)
        self.thread.start()

    def _serve(self) -> None:
        try:
            for _ in range(self.peers):
                conn, _ = self.sock.accept()
                with conn:
                    socket.send_fds(conn, [b"f"], [self.fd])
        except BaseException as e:  # noqa: BLE001 -- reported by join()
            self.error = e
        finally:
            self.sock.close()

    def join(self, timeout_s: float = 60.0) -> None:
        self.thread.join(timeout_s)
        if self.thread.is_alive() or self.error is not None:
            raise RuntimeError(f"symmetric heap descriptor exchange did not finish: {self.error}")


def _receive_fd(name: str, timeout_s: float = 60.0) -> int:
    deadline = time.monotonic() + timeout_s
    while True:
        try:
            with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as sock:
                sock.settimeout(max(1.0, deadline - time.monotonic()))
                sock.connect("\0" + name)
                _, fds, _, _ = socket.recv_fds(sock, 16, 1)
            if not fds:
                raise RuntimeError(f"no descriptor from {name}")
            return fds[0]
        except (ConnectionRefusedError, FileNotFoundError):
            if time.monotonic() > deadline:
                raise
            time.sleep(0.01)


def default_alloc() -> str:
    """``RESIHP_SYMM_ALLOC`` (``vmm`` / ``ipc``), else ``vmm`` where the driver offers it."""
    want = os.environ.get("RESIHP_SYMM_ALLOC", "")
    if want in ("vmm", "ipc"):
        return want
    return "vmm" if ext().vmm_available() else "ipc"


class SymmetricHeap:
    """``exchange(handle: bytes) -> list[bytes]`` all-gathers the IPC handles in rank order
    (``exchange_via_group`` / ``exchange_via_store``)."""

    def __init__(self, segments: dict[str, tuple[int, torch.dtype]], rank: int, world: int,
                 exchange: Callable[[bytes], list[bytes]] | None, device, abort: AbortWord | None = None,
                 _bases: list[int] | None = None, alloc: str | None = None):
        self.rank, self.world = rank, world
        self.alloc = "ipc"
        self.device = torch.device(device)
        self.dev_index = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.segments, self.pad_bytes, self.nbytes = layout(segments, world)
        check_layout(self.segments, self.pad_bytes, self.nbytes, world)
        if ext().symm_signal_bytes(world) != world * SIGNAL_SLOT_BYTES:
            raise RuntimeError("signal pad layout differs between the extension and this module")
        self.abort = abort
        self.epoch = 0
        self._opened: list[int] = []
        if _bases is not None:  # emulated ranks in one process (tests on one GPU)
            self.bases = list(_bases)
            self.local_base = self.bases[rank]
            self._owns_local = False
        else:
            self.alloc = alloc or default_alloc()
            self._owns_local = True
            if self.alloc == "vmm":
                self._map_vmm(rank, world, exchange)
            else:
                self.local_base, handle = ext().symm_alloc(self.nbytes, self.dev_index)
                handles = exchange(handle + self.signature()) if world > 1 else [handle + self.signature()]
                assert len(handles) == world
                self._check_signatures([bytes(h)[-len(self.signature()):] for h in handles])
                handles = [bytes(h)[: -len(self.signature())] for h in handles]
                self.bases = []
                for r, h in enumerate(handles):
                    if r == rank:
                        self.bases.append(self.local_base)
                    else:
                        p = ext().symm_open(h, self.dev_index)
                        self._opened.append(p)
                        self.bases.append(p)
        self.pads = torch.tensor(self.bases, dtype=torch.int64, device=self.device)
        self.status = torch.zeros(4, dtype=torch.int32, device=self.device)

    def signature(self) -> bytes:
        """16 bytes naming this heap's layout (segment names, offsets, sizes, total): every rank's
        kernels address a peer's segment at this rank's offset, so all ranks must agree."""
        import hashlib

        desc = repr((self.nbytes, self.pad_bytes, sorted((n, g.offset, g.numel, str(g.dtype))
                                                          for n, g in self.segments.items())))
        return hashlib.sha256(desc.encode()).digest()[:16]

    def _check_signatures(self, sigs: list[bytes]) -> None:
        if any(sg != sigs[self.rank] for sg in sigs):
            differ = [r for r, sg in enumerate(sigs) if sg != sigs[self.rank]]
            raise RuntimeError(f"rank {self.rank}: symmetric heap layout differs on ranks {differ}; peer "
                               "addresses would not match the peers' segments")

    def _map_vmm(self, rank: int, world: int, exchange) -> None:
        self.local_base, fd, size = ext().vmm_alloc(self.nbytes, self.dev_index)
        server = _FdServer(fd, world - 1) if world > 1 else None
        try:
            mine = json.dumps({"sock": server.name if server else "", "size": size,
                               "sig": self.signature().hex()}).encode()
            handles = exchange(mine) if world > 1 else [mine]
            assert len(handles) == world
            self._check_signatures([bytes.fromhex(json.loads(bytes(h).decode())["sig"]) for h in handles])
            self.bases = []
            for r, h in enumerate(handles):
                if r == rank:
                    self.bases.append(self.local_base)
                    continue
                peer = json.loads(bytes(h).decode())
                peer_fd = _receive_fd(peer["sock"])
                try:
                    p = ext().vmm_import(peer_fd, peer["size"], self.dev_index)
                finally:
                    os.close(peer_fd)
                self._opened.append(p)
                self.bases.append(p)
            if server is not None:
                server.join()
        finally:
            os.close(fd)

    def _unmap(self, ptr: int) -> None:
        if self.alloc == "vmm":
            ext().vmm_free(ptr, self.dev_index)
        else:
            ext().symm_close(ptr, self.dev_index)

    @classmethod
    def emulated(cls, segments: dict[str, tuple[int, torch.dtype]], world: int, device) -> list["SymmetricHeap"]:
        """``world`` heaps in one process on one device, wired as peers of each other.  Only for
        kernels that do not wait on one another (one launch per emulated rank in turn)."""
        _, _, total = layout(segments, world)
        dev = torch.device(device)
        idx = dev.index if dev.index is not None else torch.cuda.current_device()
        bases = [ext().symm_alloc(total, idx)[0] for _ in range(world)]
        heaps = [cls(segments, r, world, None, dev, _bases=bases) for r in range(world)]
        heaps[0]._emulated_bases = bases
        return heaps

    # -- views
    def tensor(self, name: str, rank: int | None = None) -> torch.Tensor:
        seg = self.segments[name]
        base = self.bases[self.rank if rank is None else rank]
        return ext().symm_tensor(base + seg.offset, seg.numel, _DTYPES[seg.dtype], self.dev_index)

    def peer_ptrs(self, name: str) -> list[int]:
        off = self.segments[name].offset
        return [b + off for b in self.bases]

    # -- synchronisation
    def barrier(self, budget_s: float = 30.0) -> None:
        """Enqueue a bounded barrier over all ranks on the current stream."""
        self.epoch += 1
        ext().symm_barrier(self.pads, self.rank, self.world, self.epoch, self.abort.dev if self.abort else 0,
                           self.status, float(budget_s))

    def restrict(self, keep: list[int]) -> None:
        """Continue with the ranks ``keep`` (old numbering, ascending) as the next generation,
        reusing every mapping: the dropped ranks' regions are unmapped, ranks are renumbered, the
        barrier epoch restarts and this rank's signal pad is cleared.  The caller makes sure every
        kept rank cleared its pad before the next barrier (a host barrier over the new group)."""
        assert self.rank in keep, "a departing rank closes its heap instead"
        bases = [self.bases[r] for r in keep]
        for r, b in enumerate(self.bases):
            if r not in keep and b in self._opened:
                torch.cuda.synchronize(self.device)
                self._unmap(b)
                self._opened.remove(b)
        self.rank, self.world, self.bases = keep.index(self.rank), len(keep), bases
        self.pads = torch.tensor(self.bases, dtype=torch.int64, device=self.device)
        ext().symm_tensor(self.local_base, self.pad_bytes, "uint8", self.dev_index).zero_()
        self.status.zero_()
        self.epoch = 0

    def validate(self) -> None:
        """Host-side invariant check: layout, distinct peer regions, pad pointers, epoch."""
        check_layout(self.segments, self.pad_bytes, self.nbytes, self.world)
        if len(self.bases) != self.world or len(set(self.bases)) != self.world or self.bases[self.rank] != self.local_base:
            raise AssertionError("peer bases are not one distinct region per rank")
        if self.pads.tolist() != self.bases:
            raise AssertionError("device pad pointers differ from the mapped bases")
        if self.epoch < 0:
            raise AssertionError("negative barrier epoch")

    def check(self) -> None:
        st = self.status.tolist()
        if st[0] == 1:
            raise PeerTimeout(f"rank {self.rank}: peer {st[1]} did not reach the barrier in time")
        if st[0] == 2 or (self.abort is not None and self.abort.raised):
            raise PeerAborted(f"rank {self.rank}: aborted by the control plane")

    def close(self) -> None:
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self._unmap(p)
        self._opened = []
        if self._owns_local and self.local_base:
            if self.alloc == "vmm":
                ext().vmm_free(self.local_base, self.dev_index)
            else:
                ext().symm_free(self.local_base, self.dev_index)
        for b in getattr(self, "_emulated_bases", []):
            ext().symm_free(b, self.dev_index)
        self._emulated_bases = []
        self.local_base = 0


def exchange_via_group(group=None) -> Callable[[bytes], list[bytes]]:
    import torch.distributed as dist

    def exchange(handle: bytes) -> list[bytes]:
        out: list = [None] * dist.get_world_size(group)
        dist.all_gather_object(out, handle, group=group)
        return out

    return exchange


def exchange_via_store(store, prefix: str, rank: int, world: int) -> Callable[[bytes], list[bytes]]:
    def exchange(handle: bytes) -> list[bytes]:
        store.set(f"{prefix}/{rank}", handle)
        return [bytes(store.get(f"{prefix}/{r}")) for r in range(world)]

    return exchange
