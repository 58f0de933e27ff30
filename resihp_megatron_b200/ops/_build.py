"""In-tree build and loading of the sm_100a kernel extension.

The extension is compiled for ``sm_100a`` only (``-gencode arch=compute_100a,code=sm_100a``)
into ``ops/_build/``.  A content hash of every source file is stored next to the shared
object, so a stale build is detected without relying on file modification times.  Loading
never falls back to a PyTorch implementation: if the extension cannot be imported the call
raises.
"""

from __future__ import annotations

import hashlib
import importlib.machinery
import importlib.util
import os
import sys
import threading
from pathlib import Path

EXT_NAME = "_rb_ops"
SRC_DIR = Path(__file__).resolve().parent / "csrc"
BUILD_DIR = Path(__file__).resolve().parent / "_build"

NVCC_FLAGS = [
    "-gencode=arch=compute_100a,code=sm_100a",
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("RB_PTXAS_VERBOSE") else "-Xptxas=-O3",
]

_lock = threading.Lock()
_module = None


def sources() -> list[Path]:
    srcs = sorted(SRC_DIR.glob("*.cu")) + [SRC_DIR / "bindings.cpp"]
    return srcs


def _hash_sources() -> str:
    h = hashlib.sha256()
    for p in sorted(SRC_DIR.iterdir()):
        if p.suffix in (".cu", ".cuh", ".cpp", ".h"):
            h.update(p.name.encode())
            h.update(p.read_bytes())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()


def _so_path() -> Path:
    return BUILD_DIR / f"{EXT_NAME}.so"


def _hash_path() -> Path:
    return BUILD_DIR / f"{EXT_NAME}.srchash"


def is_stale() -> bool:
    so, hp = _so_path(), _hash_path()
    if not so.exists() or not hp.exists():
        return True
    return hp.read_text().strip() != _hash_sources()


def build(verbose: bool = False):
    """Compile the extension for sm_100a (works without a GPU) and return the module."""
    global _module
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0a")
    os.environ.setdefault("MAX_JOBS", str(min(8, os.cpu_count() or 4)))
    from torch.utils.cpp_extension import load

    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    digest = _hash_sources()
    mod = load(
        name=EXT_NAME,
        sources=[str(s) for s in sources()],
        build_directory=str(BUILD_DIR),
        extra_cflags=["-O3", "-std=c++17"],
        extra_cuda_cflags=list(NVCC_FLAGS),
        extra_include_paths=[str(SRC_DIR)],
        extra_ldflags=["-ldl"],
        with_cuda=True,
        verbose=verbose,
    )
    _hash_path().write_text(digest)
    _module = mod
    return mod


def _import_prebuilt():
    so = _so_path()
    loader = importlib.machinery.ExtensionFileLoader(EXT_NAME, str(so))
    spec = importlib.util.spec_from_file_location(EXT_NAME, str(so), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[EXT_NAME] = mod
    return mod


def ext():
    """Return the kernel extension, building it first if it is missing or stale."""
    global _module
    if _module is not None:
        return _module
    with _lock:
        if _module is not None:
            return _module
        import torch  # noqa: F401  (loads libc10 / libtorch for the extension)

        if is_stale():
            build()
        else:
            _module = _import_prebuilt()
        return _module
