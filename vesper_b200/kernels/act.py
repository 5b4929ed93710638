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
