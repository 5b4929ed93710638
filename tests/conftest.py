"""Shared test set-up: the ``gpu`` marker, import paths and fixture loading.

``-m "not gpu"`` runs on a CPU-only machine: the oracle against the golden vectors, the host-side
contracts and the C-ABI library's exports. ``-m gpu`` runs the parity tests proper on a B200,
calling the hand-written kernels through the C ABI and checking them against the oracle.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
for path in (ROOT, ROOT / "oracle"):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200) and the built library")


def golden(name: str) -> dict[str, np.ndarray]:
    """One fixture of tests/golden/ as a dict of arrays."""
    with np.load(GOLDEN / f"{name}.npz") as data:
        return {k: data[k] for k in data.files}


def golden_names(prefix: str) -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob(f"{prefix}*.npz"))


def rel(a: np.ndarray, b: np.ndarray) -> float:
    """Relative L2 error of ``a`` against ``b`` (tests/test_delta_scan_fused.py:41-44)."""
    a64, b64 = np.asarray(a, np.float64), np.asarray(b, np.float64)
    den = np.sqrt(np.square(b64).sum())
    num = np.sqrt(np.square(a64 - b64).sum())
    return float(num / den) if den > 0 else float(num)


def max_rel(a: np.ndarray, b: np.ndarray) -> float:
    """Largest elementwise error relative to the reference's largest magnitude (normwise)."""
    a64, b64 = np.asarray(a, np.float64), np.asarray(b, np.float64)
    scale = np.abs(b64).max() if b64.size else 0.0
    err = np.abs(a64 - b64).max() if b64.size else 0.0
    return float(err / scale) if scale > 0 else float(err)


# The per-element reading of the north star's "2e-2 max relative": every element's error is
# measured against its own reference magnitude, floored at ELEM_FLOOR times the tensor's RMS, so
# an element near zero (whose absolute error is set by the magnitudes it was summed from, not by
# its own) is held to the tensor's typical scale instead of an unbounded ratio.
ELEM_FLOOR = 1.0


def elem_rel(a: np.ndarray, b: np.ndarray, floor: float = ELEM_FLOOR) -> float:
    """Largest per-element relative error ``|a - b| / max(|b|, floor * rms(b))``."""
    a64, b64 = np.asarray(a, np.float64), np.asarray(b, np.float64)
    if b64.size == 0:
        return 0.0
    rms = float(np.sqrt(np.mean(np.square(b64))))
    den = np.maximum(np.abs(b64), floor * rms)
    err = np.abs(a64 - b64)
    if rms == 0.0:
        return float(err.max())
    return float((err / den).max())


def error_report(a: np.ndarray, b: np.ndarray) -> str:
    """The three readings of one comparison as a line (relative L2, normwise max, per element)."""
    return (
        f"rel {rel(a, b):.2e} normwise {max_rel(a, b):.2e} "
        f"elem(floor rms) {elem_rel(a, b):.2e} elem(floor 0.5 rms) {elem_rel(a, b, 0.5):.2e}"
    )
