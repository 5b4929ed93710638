"""The FFN's squared ReLU as one kernel each way (the contract of ``vesper/kernels/act.py:21``).

``relu_square(z)`` is ``relu(z) ** 2`` computed as the reference's FFN computes it
(``vesper/ffn.py:44-56``: ``h = relu(z)``, then ``h * h`` in ``z``'s dtype), bit for bit, forward and
backward (``vb_relu_square_fwd`` / ``_bwd``): one pass over the hidden activations instead of the
relu, product and their backward ops.
"""

from __future__ import annotations

import torch
from torch import Tensor

from vesper_b200 import _lib
from vesper_b200.contracts import ContractError

SUPPORTED = (torch.float32, torch.bfloat16, torch.float16)


class _ReluSquare(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z):  # type: ignore[override]
        z = z.contiguous()
        y = torch.empty_like(z)
        _lib.call("vb_relu_square_fwd", z.data_ptr(), y.data_ptr(), z.numel(), _lib.DTYPE_CODE[z.dtype],
                  _lib.stream(z.device))  # fmt: skip
        ctx.save_for_backward(z)
        return y

    @staticmethod
    def backward(ctx, dy):  # type: ignore[override]
        (z,) = ctx.saved_tensors
        dy = dy.contiguous().to(z.dtype)
        dz = torch.empty_like(z)
        _lib.call("vb_relu_square_bwd", z.data_ptr(), dy.data_ptr(), dz.data_ptr(), z.numel(),
                  _lib.DTYPE_CODE[z.dtype], _lib.stream(z.device))  # fmt: skip
        return dz


def relu_square(z: Tensor) -> Tensor:
    """``relu(z) ** 2`` in ``z``'s dtype (CUDA, float32, bfloat16 or float16)."""
    if z.device.type != "cuda":
        msg = f"relu_square runs on CUDA only, got {z.device}"
        raise ContractError(msg)
    if z.dtype not in SUPPORTED:
        msg = f"z: dtype must be one of {SUPPORTED}, got {z.dtype}"
        raise ContractError(msg)
    return _ReluSquare.apply(z)


class _ResidualAdd(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, f: Tensor, keep: Tensor | None) -> Tensor:  # type: ignore[override]
        x, f = x.contiguous(), f.contiguous()
        out = torch.empty_like(x)
        width = x.shape[-1]
        k = None if keep is None else keep.contiguous()
        _lib.call("vb_residual_add", x.data_ptr(), f.data_ptr(), _lib.ptr(k), out.data_ptr(), x.numel() // width,
                  width, _lib.DTYPE_CODE[f.dtype], _lib.stream(x.device))  # fmt: skip
        ctx.keep, ctx.f_dtype, ctx.width = k, f.dtype, width
        ctx.needs = ctx.needs_input_grad
        return out

    @staticmethod
    def backward(ctx, g: Tensor):  # type: ignore[override]
        g = g.contiguous().to(torch.float32)
        dx = torch.empty_like(g) if ctx.needs[0] else None
        df = torch.empty(g.shape, dtype=ctx.f_dtype, device=g.device) if ctx.needs[1] else None
        if dx is not None or df is not None:
            _lib.call("vb_residual_add_bwd", g.data_ptr(), _lib.ptr(ctx.keep), _lib.ptr(dx), _lib.ptr(df),
                      g.numel() // ctx.width, ctx.width, _lib.DTYPE_CODE[ctx.f_dtype], _lib.stream(g.device))  # fmt: skip
        return dx, df, None


def residual_add(x: Tensor, f: Tensor, keep: Tensor | None = None) -> Tensor:
    """``x + f`` over a float32 residual stream, with the rows where ``keep [b, n]`` is False set
    to zero (as the loop zeroes halted rows), one kernel each way: the same values and gradients
    as the add followed by that zeroing. Elsewhere (not float32 CUDA, a width not a multiple of 4,
    unaligned rows) it is exactly those operations."""
    fused = (
        x.is_cuda and x.dtype == torch.float32 and f.shape == x.shape and f.dtype in SUPPORTED
        and x.shape[-1] % 4 == 0 and (keep is None or keep.shape == x.shape[:-1])
        and x.data_ptr() % 16 == 0 and f.data_ptr() % 16 == 0 and x.is_contiguous() and f.is_contiguous()
    )  # fmt: skip
    if not fused:
        out = x + f
        return out if keep is None else torch.where(keep[..., None], out, torch.zeros_like(out))
    out: Tensor = _ResidualAdd.apply(x, f, keep)
    return out
