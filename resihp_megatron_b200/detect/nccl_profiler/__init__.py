"""Build helper of the native NCCL profiler plugin (C++)."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB = HERE / "libresihp_nccl_profiler.so"


def build(out: Path | None = None) -> Path:
    """Compile the plugin (g++/c++, -Werror) and return the shared object's path."""
    cxx = shutil.which("c++") or shutil.which("g++") or shutil.which("clang++")
    if cxx is None:
        raise RuntimeError("no C++ compiler found")
    out = out or LIB
    subprocess.run([cxx, "-O2", "-fPIC", "-shared", "-std=c++17", "-Wall", "-Wextra", "-Werror", "-o", str(out),
                    str(HERE / "resihp_nccl_profiler.cpp"), "-lpthread"], check=True)
    return out
