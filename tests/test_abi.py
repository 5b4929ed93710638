"""The C-ABI library on a CPU-only machine: it loads and exports every declared entry point.

No kernel is called here (no GPU): the header ``include/vesper_b200.h`` is parsed for its
``VB_API`` declarations, and each must be exported by ``libvesper_b200.so`` and carry a ctypes
signature in ``vesper_b200._lib``.
"""

from __future__ import annotations

import ctypes
import re

from conftest import ROOT
from vesper_b200 import _lib

HEADER = ROOT / "include" / "vesper_b200.h"


def declared() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^VB_API\s+[\w\s\*]+?\b(vb_\w+)\s*\(", text, flags=re.M)


def test_the_header_declares_the_entry_points() -> None:
    names = declared()
    assert "vb_delta_scan_f32_fwd" in names
    assert "vb_keys_fwd" in names
    assert len(names) == len(set(names))


def test_the_library_loads_and_exports_every_declared_symbol() -> None:
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared():
        assert hasattr(lib, name), name


def test_every_declared_symbol_has_a_python_signature() -> None:
    assert set(declared()) == set(_lib.SIGNATURES)
    lib = _lib.load()
    assert lib.vb_abi_version() >= 1
    assert lib.vb_last_error() is not None


def test_size_queries_answer_without_a_gpu() -> None:
    assert _lib.query("vb_rms_norm_bwd_workspace", 100, 512) > 0
    assert _lib.query("vb_keys_bwd_workspace", 2, 100, 128, 2, 4) > 0
    assert _lib.query("vb_delta_scan_f32_bwd_workspace", 2, 64, 4, 64) > 0
