"""Reader of the shared-memory ring written by the NCCL profiler plugin
(``detect/nccl_profiler/``, NCCL profiler ABI v5) -- and by the device timing ring of the fused
kernels, which uses the same record format.

Ring file ``<dir>/resihp_nccl_<pid>.ring``: header ``<IIII Q>`` = (magic 0x52455348 "RESH",
version, capacity, record size, head); records ``<QQQQ iiii 24s Q>`` = (start_ns, end_ns,
comm_id, count, rank, nranks, type, peer, func, seq) where ``seq == index + 1`` marks a complete
record (seqlock).  Same format as the reference's (``resihp/detect/nccl_profile_reader.py``).
"""

from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass
from pathlib import Path

MAGIC = 0x52455348
HEADER = struct.Struct("<IIII Q")
RECORD = struct.Struct("<QQQQ iiii 24s Q")
COLL, P2P = 1 << 1, 1 << 2


@dataclass(frozen=True)
class CommRecord:
    start_ns: int
    end_ns: int
    comm_id: int
    count: int
    rank: int
    nranks: int
    type: int
    peer: int
    func: str

    @property
    def seconds(self) -> float:
        return (self.end_ns - self.start_ns) / 1e9


class RingReader:
    def __init__(self, path: str | os.PathLike):
        self.path = Path(path)
        self._f = open(self.path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        magic, _version, capacity, rsize, _ = HEADER.unpack_from(self._mm, 0)
        if magic != MAGIC or rsize != RECORD.size:
            raise ValueError(f"{path}: not a ResiHP ring (magic={magic:#x}, record={rsize} B)")
        self.capacity = capacity
        self.cursor = 0
        self.dropped = 0

    def head(self) -> int:
        return HEADER.unpack_from(self._mm, 0)[4]

    def poll(self) -> list[CommRecord]:
        head = self.head()
        if head - self.cursor > self.capacity:  # overrun: the writer lapped us
            self.dropped += head - self.cursor - self.capacity
            self.cursor = head - self.capacity
        out = []
        while self.cursor < head:
            v = RECORD.unpack_from(self._mm, HEADER.size + (self.cursor % self.capacity) * RECORD.size)
            if v[-1] != self.cursor + 1:
                break  # record still being written
            s, e, comm, count, rank, nranks, typ, peer, func, _ = v
            out.append(CommRecord(s, e, comm, count, rank, nranks, typ, peer, func.split(b"\0", 1)[0].decode()))
            self.cursor += 1
        return out

    def close(self) -> None:
        self._mm.close()
        self._f.close()


def find_rings(directory: str | os.PathLike = "/dev/shm") -> list[Path]:
    return sorted(Path(directory).glob("resihp_nccl_*.ring"))
