"""Device timing ring: fused kernels append one record per launch (earliest block start, latest
block end, from %globaltimer) to a file-backed ring in host memory that the GPU writes directly.

The file uses the NCCL profiler plugin's layout (``detect/nccl_profiler``), so
``detect.nccl_profile_reader.RingReader`` reads device records and NCCL records alike and the
fail-slow detector can consume per-kernel GPU timings without a host synchronisation.  The
reference has the NCCL half only (``resihp/detect/nccl_profiler/resihp_nccl_profiler.c``).
"""

from __future__ import annotations

import mmap
import os
import struct
from pathlib import Path

import torch

from ..detect.nccl_profile_reader import HEADER, MAGIC, RECORD
from ..ops._build import ext

VERSION = 1


class DeviceRing:
    def __init__(self, directory: str | os.PathLike | None = None, capacity: int = 4096, rank: int = 0,
                 device=None):
        if ext().ring_record_bytes() != RECORD.size:
            raise RuntimeError("device ring record layout differs from the reader's")
        d = Path(directory or os.environ.get("RESIHP_NCCL_PROF_DIR", "/dev/shm"))
        d.mkdir(parents=True, exist_ok=True)
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.path = d / f"resihp_dev_{os.getpid()}_{dev.index or 0}.ring"
        self.capacity = capacity
        self.nbytes = HEADER.size + capacity * RECORD.size
        page = mmap.PAGESIZE
        self.nbytes = (self.nbytes + page - 1) // page * page
        with open(self.path, "wb") as f:
            f.truncate(self.nbytes)
        self._f = open(self.path, "r+b")
        self._mm = mmap.mmap(self._f.fileno(), self.nbytes, access=mmap.ACCESS_WRITE)
        HEADER.pack_into(self._mm, 0, 0, VERSION, capacity, RECORD.size, 0)
        struct.pack_into("<I", self._mm, 0, MAGIC)  # magic last: a reader that sees it sees a header
        import ctypes

        self._host = ctypes.addressof(ctypes.c_char.from_buffer(self._mm))
        self.dev = ext().host_register_mapped(self._host, self.nbytes)
        self.stamp = torch.zeros(ext().kernel_stamp_bytes() // 8 + 1, dtype=torch.int64, device=dev)
        self.stamp[0] = -1  # start = max: the first block's atomicMin takes over
        self.rank = rank

    def close(self) -> None:
        if self._host:
            torch.cuda.synchronize()
            ext().host_unregister(self._host)
            self._host = 0
            del self.stamp
            self._mm.close()
            self._f.close()
