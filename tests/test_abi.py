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


def _refused(name: str, *args: object, match: str) -> None:
    """The entry point returns an error status, with ``match`` in its message, before it touches
    a pointer or launches anything (so this runs without a GPU)."""
    try:
        _lib.call(name, *args)
    except _lib.KernelError as exc:
        assert match in str(exc), str(exc)
    else:
        raise AssertionError(f"{name} accepted {args}")


def test_the_compaction_entry_points_refuse_bad_arguments_without_a_gpu() -> None:
    sizes = (ctypes.c_longlong * 1)(64)
    ptrs = (ctypes.c_void_p * 1)(None)
    _refused("vb_gather_rows_slabs", None, None, 1, 10, 10, 0, 1, ptrs, ptrs, sizes, None, match="bad shape")
    _refused("vb_gather_rows_slabs", None, None, 1, 10, 10, 4, 1, ptrs, ptrs, sizes, None, match="null index")
    _refused("vb_flatten_compaction", None, None, None, 1 << 16, 1 << 16, None, None, None, None, None, None,
             match="exceed int32")  # fmt: skip
    _refused("vb_flatten_compaction", None, None, None, 2, 8, None, None, None, None, None, None, match="null pointer")
    _refused("vb_expand_rows", None, 1 << 16, 1 << 16, 1, 1, ptrs, ptrs, ptrs, sizes, None, match="exceed int32")


def test_the_bucket_entry_points_refuse_bad_arguments_without_a_gpu() -> None:
    bodies = (ctypes.c_void_p * 24)()
    _refused("vb_slab_switch", None, 100, 0, None, bodies, match="buckets")
    _refused("vb_slab_switch", None, 1 << 30, 1, None, bodies, match="buckets")  # 31 doublings: over 24
    _refused("vb_slab_switch", None, 4096, 1024, None, bodies, match="null pointer")
    _refused("vb_slab_begin", None, None, match="null body")
    assert _lib.query("vb_slab_count", 0, 1024) == 0
    assert _lib.query("vb_slab_count", 4096, 1024) == 3
