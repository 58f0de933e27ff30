"""Worker process of the resilient GPU-runtime test: installs the PyTorch stand-ins for the
kernels (``fake_kernels``), then runs ``examples/gpu_hybrid_demo.py`` with the given arguments."""

import runpy
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from tests.helpers import fake_kernels  # noqa: E402

fake_kernels.install()
sys.argv = [str(ROOT / "examples" / "gpu_hybrid_demo.py")] + sys.argv[1:]
runpy.run_path(sys.argv[0], run_name="__main__")
