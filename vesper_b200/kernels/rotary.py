"""Rotary position embedding as one kernel each way (the op sequence of
``vesper/attention.py:178-217``, ``rotary``).

Pairs ``(x[2j], x[2j+1])`` turn by ``pos * base^(-2j/dk)``; the phases are formed in float64 and
their cosine and sine cast once to ``x``'s dtype, and every product and sum is rounded to that dtype
where the reference's separate ops round, so the result (and its gradient) equals the reference's
bit for bit. One pass over ``x`` instead of the slicing, four products, two sums and the stack.
"""

from __future__ import annotations

import torch
from torch import Tensor

from vesper_b200 import _lib
from vesper_b200.contracts import ContractError, Dims, check_shape

_FREQ: dict[tuple[int, float, torch.device], Tensor] = {}


def inv_freq(dk: int, base: float, device: torch.device) -> Tensor:
    """``base^(-2j/dk)`` for ``j < dk/2`` in float64, as the reference forms it (cached)."""
    key = (dk, float(base), device)
    f = _FREQ.get(key)
    if f is None:
        exponent = torch.arange(0, dk // 2, dtype=torch.float64, device=device) * (2.0 / dk)
        f = base ** (-exponent)
        _FREQ[key] = f
    return f


def _apply(x: Tensor, pos: Tensor, freq: Tensor, backward: bool) -> Tensor:
    b, n, heads, dk = x.shape
    y = torch.empty_like(x)
    _lib.call(
        "vb_rotary", x.data_ptr(), pos.data_ptr(), freq.data_ptr(), y.data_ptr(), b * n, heads, dk,
        int(backward), _lib.DTYPE_CODE[x.dtype], _lib.stream(x.device),
    )  # fmt: skip
    return y


class _Rotary(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, pos, freq):  # type: ignore[override]
        ctx.save_for_backward(pos, freq)
        return _apply(x.contiguous(), pos, freq, False)

    @staticmethod
    def backward(ctx, g):  # type: ignore[override]
        pos, freq = ctx.saved_tensors
        return _apply(g.contiguous(), pos, freq, True), None, None


def rotary(x: Tensor, pos: Tensor, base: float) -> Tensor:
    """``x [b, n, heads, dk]`` rotated at positions ``pos int64[b, n]`` (same shape and dtype)."""
    dims: Dims = {}
    check_shape("x", x, ("b", "n", "heads", "dk"), dims)
    check_shape("pos", pos, ("b", "n"), dims, dtype=torch.long)
    dk = dims["dk"]
    if dk % 2 != 0:
        msg = f"dk must be even for rotary pairs, got {dk}"
        raise ValueError(msg)
    if not 1.0 < base < float("inf"):
        msg = f"rotary base must be finite and above 1, got {base}"
        raise ValueError(msg)
    if x.device.type != "cuda":
        msg = f"the rotary kernel runs on CUDA only, got {x.device}"
        raise ContractError(msg)
    if dk % 8 != 0 or x.dtype not in _lib.DTYPE_CODE:
        msg = f"rotary: head dimension {dk} must be a multiple of 8 and dtype one of float32/bfloat16/float16"
        raise ContractError(msg)
    return _Rotary.apply(x, pos.contiguous(), inv_freq(dk, base, x.device))
