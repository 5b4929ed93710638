"""The head's per-token next-token loss on a B200 without float32 vocabulary copies.

PRIMITIVE ``linear_nll(x, weight, targets, *, keep_logits=False) -> [N]``: the drop-in for
``vesper/kernels/nll.py:48-169`` of mstampfli/vesper-preview, ``cross_entropy(x @ weight.T,
targets)`` per row with both gradients. The logits exist only in the matmul's own dtype (bfloat16
under CUDA autocast, as ``F.linear`` gives them), one ``[N, V]`` buffer at a time: the forward
reduces each row to its maximum ``top`` and the shifted log-sum-exp ``log sum exp(x - top)`` and its
loss ``(top - x[target]) + log_total`` (``vb_nll_row_stats``), keeping nothing ``[N, V]``; the
backward recomputes the logits with the same matmul (or takes the kept ones), overwrites them in
place with ``g * (softmax - onehot)`` computed in float32 (``vb_nll_row_grad``) and runs the two
gradient matmuls (cuBLAS), the weight's accumulated in float32. The compute dtype is the one
autocast would pick for ``F.linear`` (``vesper/kernels/nll.py:88-93``). CUDA only: the row steps
are this library's kernels; there is no CPU path.
"""

from __future__ import annotations

import torch
from torch import Tensor

from vesper_b200 import _lib
from vesper_b200.contracts import ContractError, Dims, check_ids, check_shape


def _compute_dtype(x: Tensor, weight: Tensor) -> torch.dtype:
    """What autocast would run ``F.linear(x, weight)`` in: it leaves float64 alone."""
    kind = x.device.type
    if torch.is_autocast_enabled(kind) and torch.float64 not in (x.dtype, weight.dtype):
        return torch.get_autocast_dtype(kind)
    return torch.promote_types(x.dtype, weight.dtype)


def row_stats(logits: Tensor, targets: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """``(top, log_total, nll)``, float32 ``[N]`` each, of row-strided ``logits [N, V]``."""
    n, vocab = logits.shape
    top, log_total, nll = (torch.empty(n, dtype=torch.float32, device=logits.device) for _ in range(3))
    _lib.call(
        "vb_nll_row_stats", logits.data_ptr(), logits.stride(0), targets.data_ptr(), top.data_ptr(),
        log_total.data_ptr(), nll.data_ptr(), n, vocab, _lib.DTYPE_CODE[logits.dtype], _lib.stream(logits.device),
    )  # fmt: skip
    return top, log_total, nll


def row_grad_(logits: Tensor, targets: Tensor, top: Tensor, log_total: Tensor, grad: Tensor) -> Tensor:
    """Overwrite ``logits [N, V]`` with ``grad[:, None] * (softmax - onehot)``; return it."""
    n, vocab = logits.shape
    _lib.call(
        "vb_nll_row_grad", logits.data_ptr(), logits.stride(0), targets.data_ptr(), top.data_ptr(),
        log_total.data_ptr(), grad.data_ptr(), n, vocab, _lib.DTYPE_CODE[logits.dtype], _lib.stream(logits.device),
    )  # fmt: skip
    return logits


class _LinearNLL(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, weight: Tensor, operand: Tensor, targets: Tensor, keep_logits: bool):  # type: ignore[override]
        logits = x @ operand.T
        top, log_total, nll = row_stats(logits, targets)
        ctx.save_for_backward(x, operand, targets, top, log_total, weight)
        ctx.kept = logits if keep_logits else None
        return nll

    @staticmethod
    def backward(ctx, grad: Tensor):  # type: ignore[override]
        x, operand, targets, top, log_total, weight = ctx.saved_tensors
        kept, ctx.kept = ctx.kept, None  # the first backward consumes kept logits; another recomputes
        logits = kept if kept is not None else x @ operand.T
        row_grad_(logits, targets, top, log_total, grad.to(torch.float32).contiguous())
        dx = logits @ operand
        if logits.dtype in (torch.bfloat16, torch.float16):  # the weight's accumulated in float32
            dw = torch.mm(logits.T, x, out_dtype=torch.float32)
        else:
            dw = logits.T @ x
        return dx, dw.to(weight.dtype), None, None, None


def linear_nll(x: Tensor, weight: Tensor, targets: Tensor, *, keep_logits: bool = False) -> Tensor:
    """Per-row ``-log softmax(x @ weight.T)[target]``, ``[N]`` float32.

    Args:
        x: ``[N, d]`` rows (the head's normalized inputs), on CUDA.
        weight: ``[V, d]`` the output projection (the tied embedding).
        targets: ``int32|int64 [N]`` ids in ``[0, V)``.
        keep_logits: keep the logits for the backward instead of recomputing them there.

    Raises:
        ContractError: on a shape mismatch, a target outside ``[0, V)``, a CPU tensor or an
            unsupported dtype.
    """
    dims: Dims = {}
    check_shape("x", x, ("n", "d"), dims)
    check_shape("weight", weight, ("V", "d"), dims)
    if x.device.type != "cuda":
        msg = f"the fused head loss runs on CUDA only, got x on {x.device}"
        raise ContractError(msg)
    ids = check_ids("targets", targets[None, :], ("b", "n"), dims, dims["V"])[0].to(torch.int64).contiguous()
    compute = _compute_dtype(x, weight)
    if compute not in _lib.DTYPE_CODE:
        msg = f"x: dtype must be float32, bfloat16 or float16 after autocast, got {compute}"
        raise ContractError(msg)
    operand = weight.detach().to(compute)
    out: Tensor = _LinearNLL.apply(x.to(compute), weight, operand, ids, keep_logits)
    return out
