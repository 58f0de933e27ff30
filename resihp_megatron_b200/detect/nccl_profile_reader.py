"""Reads the shared-memory ring written by the NCCL profiler plugin (``detect/nccl_profiler/``,
profiler ABI v5) and by the device timing ring of the fused kernels (same record format).

Ring format (kept identical to the reference's, ``resihp/detect/nccl_profile_reader.py``, so
the same tools read either): file ``<dir>/resihp_nccl_<pid>.ring``; a header ``<IIII Q>``
(magic ``0x52455348`` "RESH", version, capacity, record size, head) followed by ``capacity``
records ``<QQQQ iiii 24s Q>`` (start_ns, end_ns, comm_id, count, rank, nranks, type, peer,
func, seq).  A record is complete when ``seq == index + 1`` (a seqlock), so a reader never
returns a half-written record; a reader that falls more than ``capacity`` behind skips ahead
and counts what it lost.
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
        return 1e-9 * (self.end_ns - self.start_ns)

    @classmethod
    def unpack(cls, fields: tuple) -> "CommRecord":
        *numbers, name, _seq = fields
        return cls(*numbers, name.partition(b"\0")[0].decode())


class RingReader:
    def __init__(self, path: str | os.PathLike):
        self.path = Path(path)
        with open(self.path, "rb") as f:
            self._mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
        magic, _version, self.capacity, record_size, _head = HEADER.unpack_from(self._mm)
        if (magic, record_size) != (MAGIC, RECORD.size):
            self._mm.close()
            raise ValueError(f"{path}: not a ResiHP ring (magic={magic:#x}, record={record_size} B)")
        self.cursor = 0
        self.dropped = 0

    def head(self) -> int:
        return HEADER.unpack_from(self._mm)[-1]

    def _slot(self, index: int) -> tuple:
        return RECORD.unpack_from(self._mm, HEADER.size + RECORD.size * (index % self.capacity))

    def poll(self) -> list[CommRecord]:
        """Every complete record written since the last poll (oldest first)."""
        head = self.head()
        behind = head - self.cursor - self.capacity
        if behind > 0:  # the writer lapped this reader
            self.dropped += behind
            self.cursor += behind
        fresh = []
        for index in range(self.cursor, head):
            fields = self._slot(index)
            if fields[-1] != index + 1:
                break  # still being written
            fresh.append(CommRecord.unpack(fields))
        self.cursor += len(fresh)
        return fresh

    def close(self) -> None:
        self._mm.close()


def find_rings(directory: str | os.PathLike = "/dev/shm") -> list[Path]:
    return sorted(Path(directory).glob("resihp_nccl_*.ring"))
