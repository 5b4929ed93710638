"""``RMSNorm`` on a B200: one hand-written kernel per direction.

PRIMITIVE ``fused_rms_norm(x, weight, floor, eps)``: the drop-in for
``vesper/kernels/norm.py:24-52`` of mstampfli/vesper-preview (same signature, same result dtype,
the gain's gradient in the weight's dtype). Each row is divided by its largest magnitude (floored
at ``floor``) before squaring, the statistics and the gain are applied in float32 and the result
returns in ``x``'s dtype (``vesper/column.py:159-188``). The forward keeps ``inv = 1/sqrt(mean(x^2)
+ eps)`` per row; the backward is the analytic gradient with the scale held constant, the gain's
summed in a fixed order (deterministic). Kernels: ``vb_rms_norm_fwd`` / ``vb_rms_norm_bwd``.
"""

from __future__ import annotations

import torch
from torch import Tensor

from vesper_b200 import _lib
from vesper_b200.contracts import ContractError

SUPPORTED = (torch.float32, torch.bfloat16, torch.float16)


def fused_rms_norm(x: Tensor, weight: Tensor, floor: float, eps: float, out_dtype: torch.dtype | None = None) -> Tensor:
    """``[..., d] -> [..., d]`` in ``x``'s dtype; ``x`` on CUDA, ``weight [d]``.

    ``out_dtype`` (bf16 or f16, for a float32 ``x``) rounds the float32 result once to that dtype
    inside the kernel: the values and gradients of the norm followed by ``.to(out_dtype)``, with no
    float32 output tensor and no cast kernels either way."""
    if x.device.type != "cuda":
        msg = f"the fused RMSNorm runs on CUDA only, got x on {x.device}"
        raise ContractError(msg)
    if x.dtype not in SUPPORTED:
        msg = f"x: dtype must be one of {SUPPORTED}, got {x.dtype}"
        raise ContractError(msg)
    if weight.shape != (x.shape[-1],):
        msg = f"weight: expected shape ({x.shape[-1]},), got {tuple(weight.shape)}"
        raise ContractError(msg)
    if out_dtype is not None and out_dtype != x.dtype and not (
        x.dtype == torch.float32 and out_dtype in (torch.bfloat16, torch.float16)
    ):
        msg = f"out_dtype: a float32 input rounds to bf16 or f16, got {x.dtype} -> {out_dtype}"
        raise ContractError(msg)
    rows = x.reshape(-1, x.shape[-1])
    out: Tensor = _FusedRMSNorm.apply(rows, weight, floor, eps, out_dtype or x.dtype)
    return out.view(x.shape)


def rms_forward(x: Tensor, weight: Tensor, floor: float, eps: float,
                out_dtype: torch.dtype | None = None) -> tuple[Tensor, Tensor]:  # fmt: skip
    """``(y, inv)`` of row-contiguous ``x [N, d]``: ``y`` in ``out_dtype`` (default ``x``'s),
    ``inv`` float32."""
    n, width = x.shape
    dtype = out_dtype or x.dtype
    y = torch.empty(n, width, dtype=dtype, device=x.device)
    inv = torch.empty(n, dtype=torch.float32, device=x.device)
    w32 = weight.to(torch.float32).contiguous()
    _lib.call(
        "vb_rms_norm_fwd_cast", x.data_ptr(), w32.data_ptr(), y.data_ptr(), inv.data_ptr(), n, width,
        floor, eps, _lib.DTYPE_CODE[x.dtype], _lib.DTYPE_CODE[dtype], _lib.stream(x.device),
    )  # fmt: skip
    return y, inv


def rms_backward(x: Tensor, weight: Tensor, dy: Tensor, inv: Tensor) -> tuple[Tensor, Tensor]:
    """``(dx, dg)``: the input's gradient in ``x``'s dtype and the gain's in float32; ``dy`` in
    ``x``'s dtype or, for a float32 ``x``, in bf16 or f16."""
    n, width = x.shape
    dx = torch.empty_like(x)
    dg = torch.empty(width, dtype=torch.float32, device=x.device)
    w32 = weight.to(torch.float32).contiguous()
    ws = _lib.workspace(_lib.query("vb_rms_norm_bwd_workspace", n, width), x.device)
    _lib.call(
        "vb_rms_norm_bwd_cast", x.data_ptr(), w32.data_ptr(), dy.data_ptr(), inv.data_ptr(),
        dx.data_ptr(), dg.data_ptr(), ws.data_ptr(), n, width, _lib.DTYPE_CODE[x.dtype],
        _lib.DTYPE_CODE[dy.dtype], _lib.stream(x.device),
    )  # fmt: skip
    return dx, dg


class _FusedRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, floor: float, eps: float, out_dtype: torch.dtype) -> Tensor:  # type: ignore[override]
        rows = x.contiguous()
        y, inv = rms_forward(rows, weight, floor, eps, out_dtype)
        ctx.save_for_backward(rows, weight, inv)
        ctx.out_dtype = out_dtype
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        rows, weight, inv = ctx.saved_tensors
        dx, dg = rms_backward(rows, weight, dy.contiguous().to(ctx.out_dtype), inv)
        return dx, dg.to(weight.dtype), None, None, None


def add_rms_norm(x: Tensor, r: Tensor, weight: Tensor, floor: float, eps: float,
                 out_dtype: torch.dtype | None = None) -> tuple[Tensor, Tensor]:  # fmt: skip
    """``(s, y)`` with ``s = x + r`` and ``y = fused_rms_norm(s, weight, floor, eps, out_dtype)``.

    One kernel each way where ``x`` is a float32 CUDA tensor, ``r`` float32, bf16 or f16 of the
    same shape and the width a multiple of 4 up to 1024: the same values and gradients as the add
    followed by the norm (the sum is one IEEE float32 addition, as torch's mixed-dtype add makes
    it; the backward adds the sum's two gradients and rounds ``r``'s once, as autograd does).
    Elsewhere it is exactly those two operations."""
    width = x.shape[-1]
    fused = (
        x.is_cuda and x.dtype == torch.float32 and r.shape == x.shape and r.dtype in SUPPORTED
        and weight.shape == (width,) and width % 4 == 0 and width <= 1024
        and (out_dtype or x.dtype) in SUPPORTED
    )  # fmt: skip
    if not fused:
        s = x + r
        return s, fused_rms_norm(s, weight, floor, eps, out_dtype)
    s2, y2 = _AddRMSNorm.apply(x.reshape(-1, width), r.reshape(-1, width), weight, floor, eps,
                               out_dtype or x.dtype)  # fmt: skip
    return s2.view(x.shape), y2.view(x.shape)


def _aligned16(t: Tensor) -> Tensor:
    t = t.contiguous()
    return t if t.data_ptr() % 16 == 0 else t.clone()


class _AddRMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, r: Tensor, weight: Tensor, floor: float, eps: float,  # type: ignore[override]
                out_dtype: torch.dtype) -> tuple[Tensor, Tensor]:  # fmt: skip
        x, r = _aligned16(x), _aligned16(r)
        n, width = x.shape
        s = torch.empty_like(x)
        y = torch.empty(n, width, dtype=out_dtype, device=x.device)
        inv = torch.empty(n, dtype=torch.float32, device=x.device)
        w32 = _aligned16(weight.to(torch.float32))
        _lib.call(
            "vb_add_rms_norm_fwd", x.data_ptr(), r.data_ptr(), w32.data_ptr(), s.data_ptr(), y.data_ptr(),
            inv.data_ptr(), n, width, floor, eps, _lib.DTYPE_CODE[r.dtype], _lib.DTYPE_CODE[out_dtype],
            _lib.stream(x.device),
        )  # fmt: skip
        ctx.save_for_backward(s, weight, inv)
        ctx.r_dtype, ctx.out_dtype = r.dtype, out_dtype
        ctx.needs = ctx.needs_input_grad
        return s, y

    @staticmethod
    def backward(ctx, ds: Tensor | None, dy: Tensor | None):  # type: ignore[override]
        s, weight, inv = ctx.saved_tensors
        n, width = s.shape
        if dy is None:  # only the sum was read: the add's gradient alone
            d = torch.zeros_like(s) if ds is None else ds
            return d, d.to(ctx.r_dtype), None, None, None, None
        dy = _aligned16(dy.to(ctx.out_dtype))
        ds = None if ds is None else _aligned16(ds.to(torch.float32))
        dx = torch.empty_like(s)
        dr = torch.empty(n, width, dtype=ctx.r_dtype, device=s.device) if ctx.needs[1] else None
        dg = torch.empty(width, dtype=torch.float32, device=s.device)
        w32 = _aligned16(weight.to(torch.float32))
        ws = _lib.workspace(_lib.query("vb_rms_norm_bwd_workspace", n, width), s.device)
        _lib.call(
            "vb_add_rms_norm_bwd", s.data_ptr(), w32.data_ptr(), dy.data_ptr(), inv.data_ptr(), _lib.ptr(ds),
            dx.data_ptr(), _lib.ptr(dr), dg.data_ptr(), ws.data_ptr(), n, width, _lib.DTYPE_CODE[dy.dtype],
            _lib.DTYPE_CODE[ctx.r_dtype], _lib.stream(s.device),
        )  # fmt: skip
        return dx, dr, dg.to(weight.dtype), None, None, None
