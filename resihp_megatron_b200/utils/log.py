"""Process-tagged stderr logging.

Level comes from ``RESIHP_LOG_LEVEL`` (default WARNING) and the tag from ``RESIHP_WORKER_ID``
(default ``pid<N>``), so interleaved output of many ranks stays attributable (same variables
as the reference, ``resihp/utils/log.py:12-24``).
"""

from __future__ import annotations

import logging
import os
import sys
import threading

_ROOT = "resihp"
_once = threading.Lock()
_ready = False


def _configure() -> None:
    global _ready
    with _once:
        if _ready:
            return
        tag = os.environ.get("RESIHP_WORKER_ID") or f"pid{os.getpid()}"
        h = logging.StreamHandler(sys.stderr)
        h.setFormatter(logging.Formatter(f"[%(asctime)s %(levelname)s {tag} %(name)s] %(message)s"))
        root = logging.getLogger(_ROOT)
        root.addHandler(h)
        root.setLevel(os.environ.get("RESIHP_LOG_LEVEL", "WARNING").upper())
        root.propagate = False
        _ready = True


def get_logger(name: str) -> logging.Logger:
    _configure()
    if not name.startswith(_ROOT):
        name = f"{_ROOT}.{name}"
    return logging.getLogger(name)
