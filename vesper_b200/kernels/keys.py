"""``RecurrentSublayer.keys`` on a B200: the causal key filter and the key normalisation.

PRIMITIVE ``fused_keys(z, history, taps, heads)``: the drop-in for ``vesper/kernels/keys.py:28-78``
of mstampfli/vesper-preview. ``u[t] = sum_r taps[r] * z[t - r]`` with the chunk's predecessors from
``history [b, K-1, d]``, then ``normalize_keys`` per head (``vesper/recurrence.py:91-115``), float32
arithmetic, the key in ``z``'s dtype, ``[b, n, heads, d/heads]``. The backward is the reference's
own gradient (the normalisation's scale held constant, the clamp at a squared norm of one passing
gradient at and above it); the taps' gradient is summed in a fixed order and the history's is
formed only when the history requires one. The forward saves each token's normalisation
statistics (``r = 1 / max(||u||, floor)`` and the clamp decision, 8 bytes per token and head) for
the backward, which then does not recompute them. Kernels: ``vb_keys_fwd`` / ``vb_keys_bwd``.
"""

from __future__ import annotations

import torch
from torch import Tensor

from vesper_b200 import _lib
from vesper_b200.contracts import ContractError

KEY_NORM_FLOOR = 1e-6  # vesper/recurrence.py:27
SUPPORTED = (torch.float32, torch.bfloat16, torch.float16)


def _aligned(t: Tensor) -> Tensor:
    """``t`` contiguous and starting on a 16-byte boundary (the kernels' vector accesses)."""
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


def fused_keys(z: Tensor, history: Tensor, taps: Tensor, heads: int) -> Tensor:
    """Normalized keys ``[b, n, heads, d / heads]`` in ``z``'s dtype (``z [b, n, d]`` on CUDA)."""
    if z.device.type != "cuda":
        msg = f"the fused key filter runs on CUDA only, got z on {z.device}"
        raise ContractError(msg)
    if z.dtype not in SUPPORTED:
        msg = f"z: dtype must be one of {SUPPORTED}, got {z.dtype}"
        raise ContractError(msg)
    b, _, d = z.shape
    count = int(taps.shape[0])
    if taps.shape != (count, d) or history.shape != (b, count - 1, d):
        msg = f"taps {tuple(taps.shape)} / history {tuple(history.shape)} do not fit z {tuple(z.shape)}"
        raise ContractError(msg)
    out: Tensor = _FusedKeys.apply(_aligned(z), history, taps, heads)
    return out


def keys_forward(
    z: Tensor, hist: Tensor, taps: Tensor, heads: int, floor: float, stats: Tensor | None = None
) -> Tensor:
    """Keys ``[b, n, heads, d/heads]``; ``stats`` (float32 ``[b, heads, n, 2]``) receives each
    token's ``r = 1 / max(||u||, floor)`` and -1 where the clamp passes gradient (else +1)."""
    b, n, width = z.shape
    out = torch.empty(b, n, heads, width // heads, dtype=z.dtype, device=z.device)
    _lib.call(
        "vb_keys_fwd", z.data_ptr(), hist.data_ptr(), taps.data_ptr(), out.data_ptr(),
        _lib.ptr(stats), b, n, width, heads, int(taps.shape[0]), floor, _lib.DTYPE_CODE[z.dtype],
        _lib.stream(z.device),
    )  # fmt: skip
    return out


def keys_backward(
    z: Tensor,
    hist: Tensor,
    taps: Tensor,
    grad_k: Tensor,
    heads: int,
    floor: float,
    want_hist: bool,
    stats: Tensor | None = None,
) -> tuple[Tensor, Tensor, Tensor | None]:
    """Input, taps and history gradients; ``stats`` from ``keys_forward`` on the same inputs, or
    None to recompute them."""
    b, n, width = z.shape
    count = int(taps.shape[0])
    grad_z = torch.empty_like(z)
    grad_taps = torch.empty(count, width, dtype=torch.float32, device=z.device)
    grad_hist = (
        torch.empty(b, count - 1, width, dtype=torch.float32, device=z.device) if want_hist else None
    )
    ws = _lib.workspace(_lib.query("vb_keys_bwd_workspace", b, n, width, heads, count), z.device)
    _lib.call(
        "vb_keys_bwd", z.data_ptr(), hist.data_ptr(), taps.data_ptr(), grad_k.data_ptr(),
        _lib.ptr(stats), grad_z.data_ptr(), grad_taps.data_ptr(), _lib.ptr(grad_hist), ws.data_ptr(),
        b, n, width, heads, count, floor, _lib.DTYPE_CODE[z.dtype], _lib.stream(z.device),
    )  # fmt: skip
    return grad_z, grad_taps, grad_hist


class _FusedKeys(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z: Tensor, history: Tensor, taps: Tensor, heads: int) -> Tensor:  # type: ignore[override]
        hist = _aligned(history.to(torch.float32))
        wide = taps.to(torch.float32).contiguous()
        b, n, _ = z.shape
        stats = torch.empty(b, heads, n, 2, dtype=torch.float32, device=z.device)
        k = keys_forward(z, hist, wide, heads, KEY_NORM_FLOOR, stats)
        ctx.save_for_backward(z, hist, wide, stats)
        ctx.heads = heads
        ctx.history_dtype = history.dtype
        ctx.taps_dtype = taps.dtype
        return k

    @staticmethod
    def backward(ctx, grad_k: Tensor):  # type: ignore[override]
        z, hist, wide, stats = ctx.saved_tensors
        want_hist = bool(ctx.needs_input_grad[1])
        grad_z, grad_taps, grad_hist = keys_backward(
            z, hist, wide, _aligned(grad_k.to(z.dtype)), ctx.heads, KEY_NORM_FLOOR, want_hist, stats
        )
        gh = grad_hist.to(ctx.history_dtype) if grad_hist is not None else None
        return grad_z, gh, grad_taps.to(ctx.taps_dtype), None
