"""Offline install of the reference implementation into ``baseline/_ref`` (the reference arm of
``bench.py``).

    python baseline/install_reference.py [--source DIR] [--force]

Runs ``pip install --no-index --no-build-isolation --find-links /opt/wheelhouse --target
baseline/_ref <source>``; the reference declares ``torch>=2.10``, which the offline wheelhouse
cannot resolve, so on that failure the same command is repeated with ``--no-deps`` (the installed
torch is used).  The reference's ``examples/`` directory is not part of its wheel, but its chaos
benchmark starts ``examples/hetero_demo.py`` relative to the package root, so it is copied next
to the installed package unchanged.  The source defaults to a ``reference`` checkout beside this
repository; without one (e.g. on a machine that only received a copy of this tree) nothing is
done.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
TARGET = os.path.join(HERE, "_ref")
DEFAULT_SOURCE = os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
WHEELHOUSE = "/opt/wheelhouse"


def installed() -> bool:
    return os.path.isdir(os.path.join(TARGET, "resihp")) and os.path.isfile(
        os.path.join(TARGET, "examples", "hetero_demo.py"))


def install(source: str = DEFAULT_SOURCE, force: bool = False) -> str:
    """Install (idempotent); returns a one-line outcome."""
    if installed() and not force:
        return f"already installed in {TARGET}"
    if not os.path.isfile(os.path.join(source, "pyproject.toml")) and not os.path.isfile(
            os.path.join(source, "setup.py")):
        return f"no reference source at {source}; nothing installed"
    base = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links", WHEELHOUSE,
            "--target", TARGET, "--upgrade", source]
    outcome = "installed"
    proc = subprocess.run(base, capture_output=True, text=True)
    if proc.returncode != 0:
        proc = subprocess.run(base[:-1] + ["--no-deps", source], capture_output=True, text=True)
        outcome = "installed with --no-deps (dependency resolution failed offline)"
    if proc.returncode != 0:
        return "install failed: " + (proc.stderr.strip().splitlines() or ["?"])[-1]
    examples = os.path.join(source, "examples")
    if os.path.isdir(examples):
        shutil.copytree(examples, os.path.join(TARGET, "examples"), dirs_exist_ok=True)
    return f"{outcome} into {TARGET}"


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--source", default=DEFAULT_SOURCE)
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(install(args.source, args.force))


if __name__ == "__main__":
    main()
