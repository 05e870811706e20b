"""Counter of this package's kernel launches (for the benchmark's ``gpu_launches``).

Every binding call that launches kernels reports how many it launched; the count is
exact for the extension's own kernels and excludes torch/NCCL kernels.
"""
from __future__ import annotations

_COUNT = 0


def add(n: int = 1) -> None:
    global _COUNT
    _COUNT += n


def count() -> int:
    return _COUNT


def reset() -> None:
    global _COUNT
    _COUNT = 0
