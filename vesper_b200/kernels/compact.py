"""The loop's active-token bookkeeping on a B200: compaction and multi-tensor row copies.

``compact_index(active)`` packs each batch row's active tokens at the front of an index list
(``vb_compact_index``); ``gather_rows`` / ``expand_rows`` move per-token rows between the dense
``[b, n, ...]`` layout and compact buffers; ``select_rows`` is the copy-forward merge
``where(mask, fresh, carried)`` of ``vesper/column.py:140-143`` and ``vesper/loop.py:523-537`` for
every tensor of a merge in one launch. All keep static shapes (compact buffers are sized for the
worst case and the kernels read the live count on the device), so they can be captured, and all
are differentiable: each one's backward is another of them.
"""

from __future__ import annotations

import ctypes
from collections.abc import Sequence
from dataclasses import dataclass

import torch
from torch import Tensor

from vesper_b200 import _lib
from vesper_b200.contracts import ContractError

MAX_TENSORS = 12  # tensors per launch


@dataclass(frozen=True)
class Compaction:
    """One batch's active set: ``idx [b, n]`` (token of each compact row, -1 padding),
    ``rank [b, n]`` (compact row of each token, -1 if halted), ``counts [b]``, ``qpos [b, n]``
    (``idx`` plus the attention cache length), all int32 on the device, and ``active`` itself."""

    active: Tensor
    idx: Tensor
    rank: Tensor
    counts: Tensor
    qpos: Tensor
    slab_first: int = 0  # > 0: compact buffers feed bucketed work (``compact_flat``)
    relayout: Compaction | None = None  # ``compact_flat``: flat compact rows <-> per-row compact rows


def compact_index(active: Tensor, qpos_offset: int = 0) -> Compaction:
    """The compaction of ``active bool[b, n]`` (on the device, no synchronisation)."""
    if active.dtype != torch.bool or active.dim() != 2:
        msg = f"active: dtype must be torch.bool with shape [b, n], got {active.dtype} {tuple(active.shape)}"
        raise ContractError(msg)
    if active.device.type != "cuda":
        msg = f"the compaction runs on CUDA only, got {active.device}"
        raise ContractError(msg)
    active = active.contiguous()
    b, n = active.shape
    idx = torch.empty(b, n, dtype=torch.int32, device=active.device)
    rank, qpos = torch.empty_like(idx), torch.empty_like(idx)
    counts = torch.empty(b, dtype=torch.int32, device=active.device)
    _lib.call(
        "vb_compact_index", active.data_ptr(), idx.data_ptr(), rank.data_ptr(), counts.data_ptr(),
        qpos.data_ptr(), b, n, int(qpos_offset), _lib.stream(active.device),
    )  # fmt: skip
    return Compaction(active, idx, rank, counts, qpos)


def compact_flat(active: Tensor, slab_first: int) -> Compaction:
    """All ``b x n`` tokens of ``active bool[b, n]`` as ONE compact row: ``idx``, ``rank``
    ``[1, b n]`` over the flattened tokens, ``counts [1]`` the active total (on the device, no
    synchronisation); ``relayout`` moves rows between this flat compact layout and the per-row
    one of ``compact_index(active)`` (its rows ``(b, r)`` at ``b n + r``). Its compact buffers feed work cut into slabs of ``slab_first``, ``slab_first``,
    ``2 slab_first``, ... rows (``vesper_b200.kernels.slabs``): a gather zeroes its rows from the
    count to the end of the last running slab and leaves the rest, so copies follow the active
    rows, not the buffer's size."""
    if slab_first < 1:
        msg = f"slab_first must be at least 1, got {slab_first}"
        raise ContractError(msg)
    per_row = compact_index(active)
    b, n = per_row.idx.shape
    idx = torch.empty(1, b * n, dtype=torch.int32, device=active.device)
    rank, flat_pb, pb_flat = torch.empty_like(idx), torch.empty_like(idx), torch.empty_like(idx)
    counts = torch.empty(1, dtype=torch.int32, device=active.device)
    _lib.call(
        "vb_flatten_compaction", per_row.idx.data_ptr(), per_row.rank.data_ptr(), per_row.counts.data_ptr(), b, n,
        idx.data_ptr(), rank.data_ptr(), counts.data_ptr(), flat_pb.data_ptr(), pb_flat.data_ptr(),
        _lib.stream(active.device),
    )  # fmt: skip
    flat_active = per_row.active.view(1, b * n)
    # gather through it: per-row compact rows ([1, b n] = [b, n] packed per row) -> flat compact rows;
    # expand through it: the inverse (padding rows of each batch row zero)
    relayout = Compaction(flat_active, flat_pb, pb_flat, counts, flat_pb, slab_first)
    return Compaction(flat_active, idx, rank, counts, idx, slab_first, relayout)


def _row_bytes(t: Tensor, rows: int) -> int:
    return t.numel() * t.element_size() // max(rows, 1)


def _ptrs(ts: Sequence[Tensor | None]) -> ctypes.Array[ctypes.c_void_p]:
    return (ctypes.c_void_p * len(ts))(*[None if t is None else t.data_ptr() for t in ts])


def _sizes(vals: Sequence[int]) -> ctypes.Array[ctypes.c_longlong]:
    return (ctypes.c_longlong * len(vals))(*vals)


def _check_rows(name: str, ts: Sequence[Tensor | None], lead: tuple[int, int], device: torch.device) -> None:
    if not 1 <= len(ts) <= MAX_TENSORS:
        msg = f"{name}: {len(ts)} tensors, between 1 and {MAX_TENSORS} per call"
        raise ContractError(msg)
    for i, t in enumerate(ts):
        if t is None:
            continue
        if tuple(t.shape[:2]) != lead:
            msg = f"{name}[{i}]: leading axes {tuple(t.shape[:2])}, expected {lead}"
            raise ContractError(msg)
        if t.device != device:
            msg = f"{name}[{i}] is on {t.device}, the mask on {device}"
            raise ContractError(msg)


def _select(mask: Tensor, invert: bool, a: Sequence[Tensor | None], b: Sequence[Tensor | None],
            like: Sequence[Tensor]) -> list[Tensor]:  # fmt: skip
    tokens = mask.numel()
    out = [torch.empty_like(t) for t in like]
    if tokens == 0:
        return out
    _lib.call(
        "vb_select_rows", mask.data_ptr(), int(invert), len(out), _ptrs(a), _ptrs(b), _ptrs(out),
        _sizes([_row_bytes(t, tokens) for t in out]), tokens, _lib.stream(mask.device),
    )  # fmt: skip
    return out


class _Select(torch.autograd.Function):
    @staticmethod
    def forward(ctx, mask, n, *tensors):  # type: ignore[override]
        fresh, carried = tensors[:n], tensors[n:]
        ctx.save_for_backward(mask)
        ctx.n = n
        ctx.has_carried = [c is not None for c in carried]
        return tuple(_select(mask, False, fresh, carried, fresh))

    @staticmethod
    def backward(ctx, *grads):  # type: ignore[override]
        (mask,) = ctx.saved_tensors
        g = [torch.zeros_like(x) if x is None else x.contiguous() for x in grads]
        d_fresh = _select(mask, False, g, [None] * len(g), g)
        d_carried = _select(mask, True, g, [None] * len(g), g)
        d_carried = [d if has else None for d, has in zip(d_carried, ctx.has_carried, strict=True)]
        return (None, None, *d_fresh, *d_carried)


def select_rows(mask: Tensor, fresh: Sequence[Tensor], carried: Sequence[Tensor | None]) -> list[Tensor]:
    """``[where(mask, f, c) for f, c]`` per token row (``mask bool[b, n]``); ``c`` None is zero."""
    if len(fresh) != len(carried):
        msg = f"select_rows: {len(fresh)} fresh tensors, {len(carried)} carried"
        raise ContractError(msg)
    lead = (mask.shape[0], mask.shape[1])
    _check_rows("fresh", fresh, lead, mask.device)
    _check_rows("carried", carried, lead, mask.device)
    for f, c in zip(fresh, carried, strict=True):
        if c is not None and (c.shape != f.shape or c.dtype != f.dtype):
            msg = f"carried {tuple(c.shape)} {c.dtype} does not match fresh {tuple(f.shape)} {f.dtype}"
            raise ContractError(msg)
    fresh = [t.contiguous() for t in fresh]
    carried = [None if t is None else t.contiguous() for t in carried]
    return list(_Select.apply(mask.contiguous(), len(fresh), *fresh, *carried))


def _gather(comp: Compaction, src: Sequence[Tensor]) -> list[Tensor]:
    b, n = comp.idx.shape
    out = [torch.empty_like(t) for t in src]  # compact buffers sized for the worst case (n rows)
    if b * n == 0:
        return out
    if comp.slab_first > 0:  # zero padding up to the last running slab only
        _lib.call(
            "vb_gather_rows_slabs", comp.idx.data_ptr(), comp.counts.data_ptr(), b, n, n, comp.slab_first,
            len(src), _ptrs(src), _ptrs(out), _sizes([_row_bytes(t, b * n) for t in src]),
            _lib.stream(comp.idx.device),
        )  # fmt: skip
        return out
    _lib.call(
        "vb_gather_rows", comp.idx.data_ptr(), comp.counts.data_ptr(), b, n, n, len(src), _ptrs(src),
        _ptrs(out), _sizes([_row_bytes(t, b * n) for t in src]), _lib.stream(comp.idx.device),
    )  # fmt: skip
    return out


def _expand(comp: Compaction, src: Sequence[Tensor], fallback: Sequence[Tensor | None]) -> list[Tensor]:
    b, n = comp.rank.shape
    out = [torch.empty_like(t) for t in src]
    if b * n == 0:
        return out
    _lib.call(
        "vb_expand_rows", comp.rank.data_ptr(), b, n, n, len(src), _ptrs(src), _ptrs(fallback),
        _ptrs(out), _sizes([_row_bytes(t, b * n) for t in src]), _lib.stream(comp.rank.device),
    )  # fmt: skip
    return out


class _Gather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, comp, *src):  # type: ignore[override]
        ctx.comp = comp
        return tuple(_gather(comp, src))

    @staticmethod
    def backward(ctx, *grads):  # type: ignore[override]
        g = [x.contiguous() for x in grads]
        return (None, *_expand(ctx.comp, g, [None] * len(g)))


class _Expand(torch.autograd.Function):
    @staticmethod
    def forward(ctx, comp, n, *tensors):  # type: ignore[override]
        src, fallback = tensors[:n], tensors[n:]
        ctx.comp = comp
        ctx.has_fallback = [f is not None for f in fallback]
        return tuple(_expand(comp, src, fallback))

    @staticmethod
    def backward(ctx, *grads):  # type: ignore[override]
        g = [x.contiguous() for x in grads]
        d_src = _gather(ctx.comp, g)
        d_fb: list[Tensor | None] = [None] * len(g)
        if any(ctx.has_fallback):  # the halted rows' gradients go to the fallbacks
            d_fb = list(_select(ctx.comp.active, True, g, [None] * len(g), g))
            d_fb = [d if has else None for d, has in zip(d_fb, ctx.has_fallback, strict=True)]
        return (None, None, *d_src, *d_fb)


def gather_rows(comp: Compaction, dense: Sequence[Tensor]) -> list[Tensor]:
    """Each ``[b, n, ...]`` tensor's active rows packed at the front (zero padding rows; for a
    ``compact_flat`` compaction only up to the end of the last running slab)."""
    _check_rows("dense", dense, tuple(comp.idx.shape), comp.idx.device)
    return list(_Gather.apply(comp, *[t.contiguous() for t in dense]))


def expand_rows(comp: Compaction, compact: Sequence[Tensor], fallback: Sequence[Tensor | None] | None = None) -> list[Tensor]:
    """The inverse of ``gather_rows``: active rows from ``compact``, the others from ``fallback``
    (or zero)."""
    fallback = [None] * len(compact) if fallback is None else list(fallback)
    _check_rows("compact", compact, tuple(comp.idx.shape), comp.idx.device)
    _check_rows("fallback", fallback, tuple(comp.idx.shape), comp.idx.device)
    return list(_Expand.apply(comp, len(compact), *[t.contiguous() for t in compact],
                              *[None if t is None else t.contiguous() for t in fallback]))  # fmt: skip
