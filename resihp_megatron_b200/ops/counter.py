"""Host-side count of this package's kernel launches.

Every op wrapper adds the number of kernels it launched; ``bench.py`` reads the difference
across the timed region to report how many of the package's own kernels ran.
"""

_n = 0


def count(k: int) -> None:
    global _n
    _n += k


def launches() -> int:
    return _n


def reset_launches() -> None:
    global _n
    _n = 0
