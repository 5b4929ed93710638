"""The delta-rule scan on a B200: hand-written sm_100a kernels behind the reference's contract.

PRIMITIVE fused delta scan, the drop-in for ``vesper/kernels/delta_scan.py`` of
mstampfli/vesper-preview. ``delta_scan_fused`` and ``delta_scan_fused_fp32`` compute what
``vesper.recurrence.delta_scan_chunked`` computes: per head the state ``H [dk, dk]`` read as
``H^T q`` after the token's own write,

    H_t = H_{t-1} + beta_t k_t (v_t - H_{t-1}^T k_t)^T        o_t = H_t^T q_t,

forward and backward, the gradient reaching the initial state too (also when the state does not
require one: no fresh-leaf workaround is needed). Interface: ``q, k, v [b, n, h, dk]``,
``beta [b, n, h]``, ``state [b, h, dk, dk]`` float32.

``delta_scan_fused``: bfloat16 inputs, float32 state; the chunked WY form (64-token chunks) with
the intra-chunk transform and the chunk-state products on tcgen05 tensor cores, the per-chunk
states checkpointed in the forward and reused by the backward.

``delta_scan_fused_fp32``: float32 throughout, token by token (``vb_delta_scan_f32_*``).

Zero tokens return ``(q, state)`` with the same state object, as the reference does.

``from_logits=True`` takes the write strength as its logits ``W_beta x`` instead and forms
``beta = sigmoid(logits + shift)`` inside the kernels (the reference's ``write_strength``,
``vesper/recurrence.py:34-88``, with the modulator's per-token odds shift from
``modulation_shift``); the backward returns the logits' gradient. The result is bit-identical to
``torch.sigmoid`` followed by the scan: no separate sigmoid pass over beta and its gradient.
"""

from __future__ import annotations

import torch
from torch import Tensor

from vesper_b200 import _lib
from vesper_b200.contracts import ContractError, Dims, check_shape

MAX_HEAD_DIM = 256
BF16_MAX_HEAD_DIM = 128  # the chunked kernel pads the head dimension to one 128-wide tile; wider
# heads (up to MAX_HEAD_DIM) take the token-serial float32 kernel
INPUT_DTYPE = torch.bfloat16  # delta_scan_fused's q, k, v, beta
FP32_INPUT_DTYPE = torch.float32  # delta_scan_fused_fp32's q, k, v, beta
STATE_DTYPE = torch.float32


def fused_scan_available() -> bool:
    """Whether the fused scans can run here: a CUDA device and the built library."""
    if not torch.cuda.is_available():
        return False
    try:
        _lib.load()
    except OSError:
        return False
    return True


def _checked_length(
    q: Tensor, k: Tensor, v: Tensor, beta: Tensor, state: Tensor, input_dtype: torch.dtype
) -> int:
    """The one contract check of both scans (``vesper/kernels/delta_scan.py:93-119``)."""
    dims: Dims = {}
    check_shape("q", q, ("b", "n", "h", "dk"), dims, input_dtype)
    check_shape("k", k, ("b", "n", "h", "dk"), dims, input_dtype)
    check_shape("v", v, ("b", "n", "h", "dk"), dims, input_dtype)
    check_shape("beta", beta, ("b", "n", "h"), dims, input_dtype)
    check_shape("state", state, ("b", "h", "dk", "dk"), dims, STATE_DTYPE)
    if q.device.type != "cuda":
        msg = f"the fused scan runs on CUDA only, got q on {q.device}"
        raise ContractError(msg)
    for name, tensor in (("k", k), ("v", v), ("beta", beta), ("state", state)):
        if tensor.device != q.device:
            msg = f"{name} is on {tensor.device}, q on {q.device}"
            raise ContractError(msg)
    if dims["dk"] > MAX_HEAD_DIM:
        msg = f"head dimension {dims['dk']} exceeds the kernel's {MAX_HEAD_DIM}"
        raise ContractError(msg)
    return dims["n"]


def modulation_shift(logits: Tensor, m: Tensor, alpha: float) -> Tensor:
    """The per-token odds shift ``ln(1 + alpha m)`` [b, n] float32 that ``write_strength`` adds to
    the logits (``vesper/recurrence.py:34-88``), ``-inf`` where the factor is zero (an exact zero
    write and gradient). Same validation and messages as the reference."""
    if not 0.0 <= alpha < float("inf"):
        msg = f"alpha must be finite and non-negative, got {alpha}"
        raise ValueError(msg)
    dims: Dims = {}
    check_shape("logits", logits, ("b", "n", "h"), dims)
    check_shape("m", m, ("b", "n"), dims)
    factor = 1.0 + alpha * m.to(torch.float32)
    if bool((factor < 0).any().item()):
        msg = f"1 + alpha m must not be negative; alpha {alpha}, smallest m {m.min().item()}"
        raise ValueError(msg)
    return torch.where(factor > 0, torch.log(factor.clamp_min(torch.finfo(torch.float32).tiny)),
                       torch.full_like(factor, float("-inf"))).contiguous()  # fmt: skip


def _checked_shift(shift: Tensor | None, q: Tensor) -> Tensor | None:
    if shift is None:
        return None
    b, n = q.shape[0], q.shape[1]
    check_shape("shift", shift, ("b", "n"), {"b": b, "n": n}, torch.float32)
    if shift.device != q.device:
        msg = f"shift is on {shift.device}, q on {q.device}"
        raise ContractError(msg)
    return shift.contiguous()


# the device status word the bf16 scan's kernels report a timeout through (shared by the library)
status_word = _lib.status_word
check_status = _lib.check_status


# --- bfloat16, chunked on tcgen05 -------------------------------------------------------------------


def scan_bf16_forward(
    q: Tensor, k: Tensor, v: Tensor, beta: Tensor, state: Tensor, from_logits: bool = False,
    shift: Tensor | None = None,
) -> tuple[Tensor, Tensor, Tensor]:  # fmt: skip
    b, n, h, d = q.shape
    o = torch.empty_like(q)
    sn = torch.empty_like(state)
    saved = _lib.workspace(_lib.query("vb_delta_scan_bf16_saved_bytes", b, n, h, d), q.device)
    head = ("vb_delta_scan_bf16_fwd_logits", q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr(),
            _lib.ptr(shift)) if from_logits else (
            "vb_delta_scan_bf16_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr())  # fmt: skip
    _lib.call(
        *head, state.data_ptr(), o.data_ptr(), sn.data_ptr(), saved.data_ptr(),
        status_word(q.device).data_ptr(), b, n, h, d, _lib.stream(q.device),
    )  # fmt: skip
    return o, sn, saved


def scan_bf16_backward(
    q: Tensor, k: Tensor, v: Tensor, beta: Tensor, saved: Tensor, d_o: Tensor, d_sn: Tensor | None,
    from_logits: bool = False, shift: Tensor | None = None,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:  # fmt: skip
    b, n, h, d = q.shape
    dq, dk, dv, dbeta = (torch.empty_like(t) for t in (q, k, v, beta))
    ds0 = torch.empty(b, h, d, d, dtype=torch.float32, device=q.device)
    ws = _lib.workspace(_lib.query("vb_delta_scan_bf16_bwd_workspace", b, n, h, d), q.device)
    head = ("vb_delta_scan_bf16_bwd_logits", q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr(),
            _lib.ptr(shift)) if from_logits else (
            "vb_delta_scan_bf16_bwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr())  # fmt: skip
    _lib.call(
        *head, saved.data_ptr(), d_o.data_ptr(), _lib.ptr(d_sn), dq.data_ptr(), dk.data_ptr(),
        dv.data_ptr(), dbeta.data_ptr(), ds0.data_ptr(), ws.data_ptr(),
        status_word(q.device).data_ptr(), b, n, h, d, _lib.stream(q.device),
    )  # fmt: skip
    return dq, dk, dv, dbeta, ds0


class _ScanBF16(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q: Tensor, k: Tensor, v: Tensor, beta: Tensor, state: Tensor, from_logits: bool,  # type: ignore[override]
                shift: Tensor | None):  # fmt: skip
        q, k, v, beta, state = (t.contiguous() for t in (q, k, v, beta, state))
        o, sn, saved = scan_bf16_forward(q, k, v, beta, state, from_logits, shift)
        ctx.from_logits = from_logits
        if any(ctx.needs_input_grad):
            ctx.save_for_backward(q, k, v, beta, saved, shift)
        return o, sn

    @staticmethod
    def backward(ctx, d_o: Tensor | None, d_sn: Tensor | None):  # type: ignore[override]
        q, k, v, beta, saved, shift = ctx.saved_tensors
        d_o = torch.zeros_like(q) if d_o is None else d_o.contiguous().to(torch.bfloat16)
        d_sn = None if d_sn is None else d_sn.contiguous().to(torch.float32)
        grads = scan_bf16_backward(q, k, v, beta, saved, d_o, d_sn, ctx.from_logits, shift)
        return (*grads, None, None)


def delta_scan_fused(
    q: Tensor, k: Tensor, v: Tensor, beta: Tensor, state: Tensor, *, from_logits: bool = False,
    shift: Tensor | None = None,
) -> tuple[Tensor, Tensor]:  # fmt: skip
    """Apply ``n`` tokens to the state with the chunked bfloat16 kernels (the reference's form).

    Args:
        q: ``[b, n, h, dk]`` queries, bfloat16, on a CUDA device.
        k: ``[b, n, h, dk]`` keys, bfloat16, L2 norm at most one.
        v: ``[b, n, h, dk]`` values, bfloat16.
        beta: ``[b, n, h]`` write strengths in [0, 1], bfloat16 (their logits with ``from_logits``).
        state: ``[b, h, dk, dk]`` the state before the first token, float32.
        from_logits: ``beta`` holds the logits; the kernels form ``sigmoid(beta + shift)``.
        shift: optional ``[b, n]`` float32 per-token shift of the logits (``modulation_shift``).

    Returns:
        ``(o, state_n)``: ``o [b, n, h, dk]`` in bfloat16 and the state after the last token in
        float32. With no tokens, the empty query tensor and the unchanged state.

    Head dimensions up to 128 that are multiples of 8 run the chunked tcgen05 kernels; the others
    the contract allows (up to 256) run the token-serial float32 kernels on float32 copies.

    Raises:
        ContractError: on a shape, dtype or device mismatch, or a head dimension above 256.
    """
    if _checked_length(q, k, v, beta, state, INPUT_DTYPE) == 0:
        return q, state
    if shift is not None and not from_logits:
        msg = "shift applies to write-strength logits: pass from_logits=True"
        raise ContractError(msg)
    if q.shape[-1] > BF16_MAX_HEAD_DIM or q.shape[-1] % 8 != 0:
        # head dimensions the chunked tiles do not take (above 128, or not a multiple of 8; the
        # contract allows up to 256): the token-serial float32 kernel on float32 copies of the
        # inputs, the output back in bfloat16 (exact float32 arithmetic, slower per token)
        f32 = torch.float32
        o, sn = delta_scan_fused_fp32(q.to(f32), k.to(f32), v.to(f32), beta.to(f32), state, from_logits=from_logits,
                                      shift=shift)  # fmt: skip
        return o.to(INPUT_DTYPE), sn
    o, sn = _ScanBF16.apply(q, k, v, beta, state, bool(from_logits), _checked_shift(shift, q))
    return o, sn


# --- float32, token-serial ----------------------------------------------------------------------


def scan_f32_forward(
    q: Tensor, k: Tensor, v: Tensor, beta: Tensor, state: Tensor, keep_resid: bool, from_logits: bool = False,
    shift: Tensor | None = None,
) -> tuple[Tensor, Tensor, Tensor | None]:  # fmt: skip
    b, n, h, d = q.shape
    o = torch.empty_like(q)
    sn = torch.empty_like(state)
    resid = torch.empty_like(v) if keep_resid else None
    head = ("vb_delta_scan_f32_fwd_logits", q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr(),
            _lib.ptr(shift)) if from_logits else (
            "vb_delta_scan_f32_fwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr())  # fmt: skip
    _lib.call(
        *head, state.data_ptr(), o.data_ptr(), sn.data_ptr(), _lib.ptr(resid), b, n, h, d,
        _lib.stream(q.device),
    )  # fmt: skip
    return o, sn, resid


def scan_f32_backward(
    q: Tensor, k: Tensor, v: Tensor, beta: Tensor, state: Tensor, resid: Tensor,
    d_o: Tensor, d_sn: Tensor | None, from_logits: bool = False, shift: Tensor | None = None,
) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:  # fmt: skip
    b, n, h, d = q.shape
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dbeta, ds0 = torch.empty_like(beta), torch.empty_like(state)
    ws = _lib.workspace(_lib.query("vb_delta_scan_f32_bwd_workspace", b, n, h, d), q.device)
    head = ("vb_delta_scan_f32_bwd_logits", q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr(),
            _lib.ptr(shift)) if from_logits else (
            "vb_delta_scan_f32_bwd", q.data_ptr(), k.data_ptr(), v.data_ptr(), beta.data_ptr())  # fmt: skip
    _lib.call(
        *head, state.data_ptr(), resid.data_ptr(), d_o.data_ptr(), _lib.ptr(d_sn), dq.data_ptr(),
        dk.data_ptr(), dv.data_ptr(), dbeta.data_ptr(), ds0.data_ptr(), ws.data_ptr(), b, n, h, d,
        _lib.stream(q.device),
    )  # fmt: skip
    return dq, dk, dv, dbeta, ds0


class _ScanF32(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q: Tensor, k: Tensor, v: Tensor, beta: Tensor, state: Tensor, from_logits: bool,  # type: ignore[override]
                shift: Tensor | None):  # fmt: skip
        q, k, v, beta, state = (t.contiguous() for t in (q, k, v, beta, state))
        keep = any(ctx.needs_input_grad)
        o, sn, resid = scan_f32_forward(q, k, v, beta, state, keep, from_logits, shift)
        ctx.from_logits = from_logits
        if keep:
            ctx.save_for_backward(q, k, v, beta, state, resid, shift)
        return o, sn

    @staticmethod
    def backward(ctx, d_o: Tensor | None, d_sn: Tensor | None):  # type: ignore[override]
        q, k, v, beta, state, resid, shift = ctx.saved_tensors
        d_o = torch.zeros_like(q) if d_o is None else d_o.contiguous().to(torch.float32)
        d_sn = None if d_sn is None else d_sn.contiguous().to(torch.float32)
        grads = scan_f32_backward(q, k, v, beta, state, resid, d_o, d_sn, ctx.from_logits, shift)
        return (*grads, None, None)


def delta_scan_fused_fp32(
    q: Tensor, k: Tensor, v: Tensor, beta: Tensor, state: Tensor, *, from_logits: bool = False,
    shift: Tensor | None = None,
) -> tuple[Tensor, Tensor]:  # fmt: skip
    """Apply ``n`` tokens to the state in float32 (the reference's precision).

    Returns ``(o [b, n, h, dk], state_n)`` in float32; with no tokens, ``(q, state)``.
    ``from_logits`` / ``shift``: as for ``delta_scan_fused``.

    Raises:
        ContractError: on a shape, dtype or device mismatch, or a head dimension above 256.
    """
    if _checked_length(q, k, v, beta, state, FP32_INPUT_DTYPE) == 0:
        return q, state
    if shift is not None and not from_logits:
        msg = "shift applies to write-strength logits: pass from_logits=True"
        raise ContractError(msg)
    o, sn = _ScanF32.apply(q, k, v, beta, state, bool(from_logits), _checked_shift(shift, q))
    return o, sn


# --- one token, in place (the decode step) ---------------------------------------------------------


def delta_scan_step_(
    q: Tensor, k: Tensor, v: Tensor, beta: Tensor, state: Tensor, *, from_logits: bool = False,
    shift: Tensor | None = None,
) -> Tensor:  # fmt: skip
    """One token per (batch, head) applied to ``state`` IN PLACE; returns ``o``.

    ``delta_scan_step`` of ``vesper/recurrence.py:143-163`` batched for a decode step:
    ``H' = H + beta k (v - H^T k)^T``, ``o = H'^T q``. ``q, k, v [b, 1, h, dk]`` (or
    ``[b, h, dk]``) and ``beta [b, 1, h]`` in float32 or bfloat16 (``from_logits``: the logits,
    ``shift [b, 1]`` optional), ``state [b, h, dk, dk]`` float32, contiguous; ``o`` has ``q``'s
    shape and dtype. No autograd: the decode step's carried state is updated where it lies.
    """
    dt = q.dtype
    if dt not in (torch.float32, torch.bfloat16):
        msg = f"q: dtype must be float32 or bfloat16, got {dt}"
        raise ContractError(msg)
    b, h, d = q.shape[0], q.shape[-2], q.shape[-1]
    if q.numel() != b * h * d or k.numel() != b * h * d or v.numel() != b * h * d or beta.numel() != b * h:
        msg = f"delta_scan_step_: one token per row and head expected, got q {tuple(q.shape)}"
        raise ContractError(msg)
    check_shape("state", state, ("b", "h", "dk", "dk"), {"b": b, "h": h, "dk": d}, STATE_DTYPE)
    if not state.is_contiguous():
        msg = "state must be contiguous (it is updated in place)"
        raise ContractError(msg)
    qc, kc, vc, bc = (t.to(dt).contiguous() for t in (q, k, v, beta))
    sh = None if shift is None else shift.to(torch.float32).contiguous()
    o = torch.empty_like(qc)
    _lib.call(
        "vb_delta_scan_step", qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), bc.data_ptr(), _lib.ptr(sh),
        1 if from_logits else 0, state.data_ptr(), state.data_ptr(), o.data_ptr(), b, h, d, _lib.DTYPE_CODE[dt],
        _lib.stream(q.device),
    )  # fmt: skip
    return o
