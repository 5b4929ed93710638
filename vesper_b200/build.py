"""Build ``libvesper_b200.so`` in-tree for sm_100a (nvcc cross-compiles without a GPU)."""

from __future__ import annotations

import os
import subprocess
from pathlib import Path

CSRC = Path(__file__).resolve().parent / "csrc"
LIB = Path(__file__).resolve().parent / "libvesper_b200.so"


def build(jobs: int | None = None) -> Path:
    """Compile every CUDA source with ``-gencode arch=compute_100a,code=sm_100a``; returns the path."""
    jobs = jobs or max(1, min(16, os.cpu_count() or 1))
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", str(CSRC)], check=True)
    return LIB


if __name__ == "__main__":
    print(build())
