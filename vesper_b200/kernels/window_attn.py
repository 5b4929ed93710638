"""Sliding-window attention on a B200: hand-written sm_100a kernels behind the reference's contract.

PRIMITIVE ``window_attention(q, keys, values, window)``, the drop-in for
``vesper/kernels/window_attn.py:27-39`` of mstampfli/vesper-preview: the outputs of the ``n`` newest
of ``m + n`` consecutive key positions (the cache's ``m`` rows, then the chunk's ``n``), each
query at index ``i`` attending the keys at ``[i - window + 1, i]``, scale ``1 / sqrt(dk)``,
grouped KV heads (query head ``h`` reads key head ``h // (h_q / hkv)``): what
``WindowedAttention.attend`` (``vesper/attention.py:340-407``) computes with its blocked, masked
``scaled_dot_product_attention``. The reference pads the cache rows with zero queries for its
library kernel; these kernels take the ``m`` cache rows directly and compute only the ``n`` queries.

``window_attention_active(q, qpos, counts, keys, values, window)`` is the loop's compacted form:
``q [b, nq, h, dk]`` holds only the active tokens of each batch row, ``qpos [b, nq]`` (int32,
ascending along a row) their key indices, ``counts [b]`` (int32, on the device) how many rows of
each batch are live. Padding rows get zero output and no gradient, so buffers sized for the worst
case keep a captured graph's shapes static while the kernels read the live count.

Forward and backward run on tcgen05 tensor cores (``vb_window_attn_fwd`` / ``_bwd``): online
softmax in float32 over 128-key tiles, deterministic gradients (no atomics), for bfloat16 or
float16 inputs, as the reference's kernel path takes. float32 inputs (the reference's float32
path, its blocked masked softmax) run on CUDA cores in float32 FFMA arithmetic through the same
entry points, so float32 parity holds at float32 rounding.
"""

from __future__ import annotations

import torch
from torch import Tensor

from vesper_b200 import _lib
from vesper_b200.contracts import ContractError, Dims, check_shape, require_cuda

WINDOW_DTYPES = (torch.bfloat16, torch.float16, torch.float32)
MAX_HEAD_DIM = 128


def _check(
    q: Tensor, keys: Tensor, values: Tensor, window: int, qpos: Tensor | None, counts: Tensor | None
) -> Dims:
    dims: Dims = {}
    check_shape("q", q, ("b", "n", "h", "dk"), dims)
    check_shape("keys", keys, ("b", "l", "hkv", "dk"), dims)
    check_shape("values", values, ("b", "l", "hkv", "dk"), dims)
    if q.dtype not in WINDOW_DTYPES:
        msg = f"q: dtype must be one of {WINDOW_DTYPES}, got {q.dtype}"
        raise ContractError(msg)
    for name, t in (("keys", keys), ("values", values)):
        if t.dtype != q.dtype:
            msg = f"{name}: dtype must be {q.dtype} (q's), got {t.dtype}"
            raise ContractError(msg)
    if qpos is not None:
        check_shape("qpos", qpos, ("b", "n"), dims, torch.int32)
    if counts is not None:
        check_shape("counts", counts, ("b",), dims, torch.int32)
    require_cuda("window attention", q, keys=keys, values=values, qpos=qpos, counts=counts)
    h, hkv, dk = dims["h"], dims["hkv"], dims["dk"]
    if h % hkv != 0:
        msg = f"{h} query heads are not a multiple of {hkv} key heads"
        raise ContractError(msg)
    if dk % 16 != 0 or dk > MAX_HEAD_DIM:
        msg = f"head dimension {dk} must be a multiple of 16 and not exceed {MAX_HEAD_DIM}"
        raise ContractError(msg)
    if window < 1:
        msg = f"window {window} must be at least 1"
        raise ContractError(msg)
    if qpos is None and dims["l"] < dims["n"]:
        msg = f"keys hold {dims['l']} positions, fewer than the {dims['n']} queries"
        raise ContractError(msg)
    return dims


def attn_forward(
    q: Tensor, keys: Tensor, values: Tensor, window: int, qpos: Tensor | None, counts: Tensor | None
) -> tuple[Tensor, Tensor]:
    """``(o, lse)``: the outputs and the saved base-2 log-sum-exp ``[b, h, n]`` float32."""
    b, n, h, dk = q.shape
    length, hkv = keys.shape[1], keys.shape[2]
    o = torch.empty_like(q)
    lse = torch.empty(b, h, n, dtype=torch.float32, device=q.device)
    _lib.call(
        "vb_window_attn_fwd", q.data_ptr(), _lib.ptr(qpos), _lib.ptr(counts), keys.data_ptr(),
        values.data_ptr(), o.data_ptr(), lse.data_ptr(), _lib.status_word(q.device).data_ptr(),
        b, n, length, h, hkv, dk, window, _lib.DTYPE_CODE[q.dtype], _lib.stream(q.device),
    )  # fmt: skip
    return o, lse


def attn_backward(
    q: Tensor, keys: Tensor, values: Tensor, o: Tensor, lse: Tensor, d_o: Tensor, window: int,
    qpos: Tensor | None, counts: Tensor | None,
) -> tuple[Tensor, Tensor, Tensor]:  # fmt: skip
    """``(dq, dkeys, dvalues)`` of ``sum(o * d_o)``."""
    b, n, h, dk = q.shape
    length, hkv = keys.shape[1], keys.shape[2]
    dq, dkeys, dvalues = torch.empty_like(q), torch.empty_like(keys), torch.empty_like(values)
    ws = _lib.workspace(_lib.query("vb_window_attn_bwd_workspace", b, n, h), q.device)
    _lib.call(
        "vb_window_attn_bwd", q.data_ptr(), _lib.ptr(qpos), _lib.ptr(counts), keys.data_ptr(),
        values.data_ptr(), o.data_ptr(), lse.data_ptr(), d_o.data_ptr(), dq.data_ptr(),
        dkeys.data_ptr(), dvalues.data_ptr(), ws.data_ptr(), _lib.status_word(q.device).data_ptr(),
        b, n, length, h, hkv, dk, window, _lib.DTYPE_CODE[q.dtype], _lib.stream(q.device),
    )  # fmt: skip
    return dq, dkeys, dvalues


class _WindowAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, keys, values, qpos, counts, window):  # type: ignore[override]
        q, keys, values = (t.contiguous() for t in (q, keys, values))
        o, lse = attn_forward(q, keys, values, window, qpos, counts)
        ctx.window = window
        ctx.save_for_backward(q, keys, values, o, lse, qpos, counts)
        return o

    @staticmethod
    def backward(ctx, d_o):  # type: ignore[override]
        q, keys, values, o, lse, qpos, counts = ctx.saved_tensors
        d_o = d_o.contiguous().to(q.dtype)
        dq, dk, dv = attn_backward(q, keys, values, o, lse, d_o, ctx.window, qpos, counts)
        return dq, dk, dv, None, None, None


def window_attention(q: Tensor, keys: Tensor, values: Tensor, window: int) -> Tensor:
    """Outputs ``[b, n, h, dk]`` of ``q`` over ``keys, values [b, m + n, hkv, dk]`` (cache first).

    Raises:
        ContractError: on a shape, dtype or device mismatch, a head dimension that is not a
            multiple of 16 up to 128, or fewer key positions than queries.
    """
    dims = _check(q, keys, values, window, None, None)
    if dims["n"] == 0 or dims["b"] == 0:
        return q.new_zeros(q.shape)
    return _WindowAttention.apply(q, keys, values, None, None, int(window))


def window_attention_active(
    q: Tensor, qpos: Tensor, counts: Tensor | None, keys: Tensor, values: Tensor, window: int
) -> Tensor:
    """The compacted form: outputs ``[b, nq, h, dk]`` of the live query rows (zero for padding).

    Args:
        q: ``[b, nq, h, dk]`` the active tokens' queries, packed at the front of each batch row.
        qpos: ``[b, nq]`` int32 key index of each query row, ascending along a batch row.
        counts: ``[b]`` int32 live rows per batch row (None: all ``nq``); read on the device.
        keys, values: ``[b, l, hkv, dk]`` every position's keys and values.
        window: keys ``(qpos - window, qpos]`` are attended.
    """
    dims = _check(q, keys, values, window, qpos, counts)
    if dims["n"] == 0 or dims["b"] == 0:
        return q.new_zeros(q.shape)
    qpos = qpos.contiguous()
    counts = None if counts is None else counts.contiguous()
    return _WindowAttention.apply(q, keys, values, qpos, counts, int(window))
