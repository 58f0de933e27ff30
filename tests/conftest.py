"""Shared pytest configuration.

Markers: ``gpu`` (needs a CUDA device; runs on a B200), ``dist`` (spawns local processes
over gloo), ``slow`` (long-running).  GPU tests are skipped automatically when no CUDA
device is visible, so ``pytest -m "not gpu"`` and a plain run both pass on a CPU host.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a)")
    config.addinivalue_line("markers", "multigpu: needs two or more CUDA GPUs")
    config.addinivalue_line("markers", "dist: multi-process test over gloo on localhost")
    config.addinivalue_line("markers", "slow: long-running test")


def pytest_collection_modifyitems(config, items):
    try:
        import torch

        n = torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:  # pragma: no cover
        n = 0
    skip_gpu = pytest.mark.skip(reason="no CUDA device")
    skip_multi = pytest.mark.skip(reason="needs >= 2 CUDA devices")
    for item in items:
        if "gpu" in item.keywords and n == 0:
            item.add_marker(skip_gpu)
        if "multigpu" in item.keywords and n < 2:
            item.add_marker(skip_multi)


@pytest.fixture
def store():
    """A master ``TCPStore`` on 127.0.0.1 for multi-process tests; yields ``(host, port)``."""
    import torch.distributed as dist

    srv = dist.TCPStore("127.0.0.1", 0, is_master=True, wait_for_workers=False)
    yield ("127.0.0.1", srv.port)
    del srv


@pytest.fixture(autouse=True)
def _clear_kernel_error_word(request):
    """GPU tests start with a clean per-device kernel error word, so a bounded wait that ran out
    in one test is reported by that test and not by the next one that checks the word."""
    if "gpu" in request.keywords:
        try:
            import torch

            if torch.cuda.is_available():
                from resihp_megatron_b200.ops import error_state

                error_state().zero_()
        except Exception:  # noqa: BLE001 -- the extension may not be built on this host
            pass
    yield
