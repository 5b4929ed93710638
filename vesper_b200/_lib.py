"""ctypes binding of libvesper_b200.so, the package's hand-written sm_100a kernels.

The library is a plain C ABI (``include/vesper_b200.h``): device pointers, sizes and a CUDA stream.
This module loads it once, declares every entry point's argument types and turns a non-zero
status into an exception carrying the library's own message. There is no fallback: if the library
is missing or a kernel fails, the call raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

LIB_PATH = Path(os.environ.get("VESPER_B200_LIB", Path(__file__).resolve().parent / "libvesper_b200.so"))

VB_F32, VB_BF16, VB_F16 = 0, 1, 2
DTYPE_CODE = {torch.float32: VB_F32, torch.bfloat16: VB_BF16, torch.float16: VB_F16}

_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_F = ctypes.c_float
_SZ = ctypes.c_size_t

# entry point -> (restype, argtypes); the single source of the Python-side signatures
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "vb_last_error": (ctypes.c_char_p, []),
    "vb_abi_version": (_I, []),
    "vb_launch_count": (ctypes.c_ulonglong, []),
    "vb_rms_norm_fwd": (_I, [_P, _P, _P, _P, _I64, _I, _F, _F, _I, _P]),
    "vb_rms_norm_bwd_workspace": (_SZ, [_I64, _I]),
    "vb_rms_norm_bwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _I64, _I, _I, _P]),
    "vb_rms_norm_bwd_noalloc": (_I, [_P, _P, _P, _P, _P, _P, _I64, _I, _I, _P]),
    "vb_rms_norm_fwd_cast": (_I, [_P, _P, _P, _P, _I64, _I, _F, _F, _I, _I, _P]),
    "vb_rms_norm_bwd_cast": (_I, [_P, _P, _P, _P, _P, _P, _P, _I64, _I, _I, _I, _P]),
    "vb_add_rms_norm_fwd": (_I, [_P] * 6 + [_I64, _I, _F, _F, _I, _I, _P]),
    "vb_add_rms_norm_bwd": (_I, [_P] * 9 + [_I64, _I, _I, _I, _P]),
    "vb_keys_fwd": (_I, [_P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _I, _P]),
    "vb_keys_bwd_workspace": (_SZ, [_I, _I, _I, _I, _I]),
    "vb_keys_bwd": (_I, [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I, _I, _F, _I, _P]),
    "vb_delta_scan_f32_fwd": (_I, [_P] * 8 + [_I, _I, _I, _I, _P]),
    "vb_delta_scan_f32_bwd_workspace": (_SZ, [_I, _I, _I, _I]),
    "vb_delta_scan_f32_bwd": (_I, [_P] * 14 + [_I, _I, _I, _I, _P]),
    "vb_delta_scan_bf16_saved_bytes": (_SZ, [_I, _I, _I, _I]),
    "vb_delta_scan_bf16_fwd": (_I, [_P] * 9 + [_I, _I, _I, _I, _P]),
    "vb_delta_scan_bf16_bwd_workspace": (_SZ, [_I, _I, _I, _I]),
    "vb_delta_scan_bf16_bwd": (_I, [_P] * 14 + [_I, _I, _I, _I, _P]),
    "vb_nll_row_stats": (_I, [_P, _I64, _P, _P, _P, _P, _I64, _I, _I, _P]),
    "vb_ring_attend_workspace": (_SZ, [_I, _I, _I, _I, _I]),
    "vb_ring_attend": (_I, [_P] * 10 + [_I] * 7 + [_P]),
    "vb_delta_scan_step": (_I, [_P, _P, _P, _P, _P, _I, _P, _P, _P, _I, _I, _I, _I, _P]),
    "vb_nll_row_grad": (_I, [_P, _I64, _P, _P, _P, _P, _I64, _I, _I, _P]),
    "vb_delta_scan_f32_fwd_logits": (_I, [_P] * 9 + [_I, _I, _I, _I, _P]),
    "vb_delta_scan_f32_bwd_logits": (_I, [_P] * 15 + [_I, _I, _I, _I, _P]),
    "vb_delta_scan_bf16_fwd_logits": (_I, [_P] * 10 + [_I, _I, _I, _I, _P]),
    "vb_delta_scan_bf16_bwd_logits": (_I, [_P] * 15 + [_I, _I, _I, _I, _P]),
    "vb_window_attn_fwd": (_I, [_P] * 8 + [_I] * 8 + [_P]),
    "vb_window_attn_bwd_workspace": (_SZ, [_I, _I, _I]),
    "vb_window_attn_bwd": (_I, [_P] * 13 + [_I] * 8 + [_P]),
    "vb_compact_index": (_I, [_P] * 5 + [_I, _I, _I, _P]),
    "vb_select_rows": (_I, [_P, _I, _I, _P, _P, _P, _P, ctypes.c_longlong, _P]),
    "vb_gather_rows": (_I, [_P, _P, _I, _I, _I, _I, _P, _P, _P, _P]),
    "vb_expand_rows": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P]),
    "vb_gather_rows_slabs": (_I, [_P, _P, _I, _I, _I, _I, _I, _P, _P, _P, _P]),
    "vb_flatten_compaction": (_I, [_P, _P, _P, _I, _I, _P, _P, _P, _P, _P, _P]),
    "vb_slab_count": (_I, [_I, _I]),
    "vb_slab_switch": (_I, [_P, _I, _I, _P, _P]),
    "vb_slab_begin": (_I, [_P, _P]),
    "vb_slab_close": (_I, [_P]),
    "vb_relu_square_fwd": (_I, [_P, _P, ctypes.c_longlong, _I, _P]),
    "vb_relu_square_bwd": (_I, [_P, _P, _P, ctypes.c_longlong, _I, _P]),
    "vb_rotary": (_I, [_P, _P, _P, _P, ctypes.c_longlong, _I, _I, _I, _I, _P]),
    "vb_residual_add": (_I, [_P, _P, _P, _P, ctypes.c_longlong, _I, _I, _P]),
    "vb_residual_add_bwd": (_I, [_P, _P, _P, _P, ctypes.c_longlong, _I, _I, _P]),
}


class KernelError(RuntimeError):
    """A kernel entry point returned an error status."""


_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """The loaded library; raises ``OSError`` if it was not built (``vesper_b200.build``)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            msg = f"{LIB_PATH} is missing: build it with `python -c 'import vesper_b200.build as b; b.build()'`"
            raise OSError(msg)
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
    return _lib


def call(name: str, *args: object) -> None:
    """Call entry point ``name``; raise ``KernelError`` with the library's message on failure."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != 0:
        message = lib.vb_last_error().decode(errors="replace")
        raise KernelError(f"{name}: {message} (status {status})")


def query(name: str, *args: object) -> int:
    """Call a size query entry point."""
    return int(getattr(load(), name)(*args))


def launch_count() -> int:
    """Kernels the library has launched so far in this process."""
    return int(load().vb_launch_count())


def ptr(t: torch.Tensor | None) -> int | None:
    """The device address of ``t`` (None for a missing optional tensor)."""
    return None if t is None else t.data_ptr()


def stream(device: torch.device) -> int:
    """torch's current CUDA stream on ``device`` as a raw handle."""
    return torch.cuda.current_stream(device).cuda_stream


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Scratch memory from torch's caching allocator (graph-capturable, never cudaMalloc here)."""
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


# --- device status word ----------------------------------------------------------------------------

_STATUS: dict[torch.device, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """The int32 the tensor-core kernels OR an error bit into (a bounded wait that gave up)."""
    word = _STATUS.get(device)
    if word is None:
        word = torch.zeros(1, dtype=torch.int32, device=device)
        _STATUS[device] = word
    return word


def check_status(device: torch.device) -> None:
    """Synchronise and raise if a kernel on ``device`` reported a timeout (never under capture)."""
    word = _STATUS.get(device)
    if word is not None and int(word.item()) != 0:
        value = int(word.item())
        word.zero_()
        msg = f"a kernel gave up waiting on the tensor core or a copy (status {value})"
        raise KernelError(msg)
