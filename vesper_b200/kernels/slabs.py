"""Per-token work over the active rows only, inside one captured graph.

After the loop's first passes most tokens have halted (config 4 at random initialisation: about
92 % after two passes), yet a dense pass still runs the feed-forward block over all ``b x n`` rows;
the reference does the same and notes that "a kernel skips them" (``vesper/loop.py:24-26``). Here
the active rows are packed at the front of a buffer of ``cap`` rows (``compact_flat``) and the work
runs over a prefix of it, a bucket ``[0, end_k)`` with ``end_k = first * 2^k`` (the last clamped to
``cap``): the smallest bucket that holds the count. ``run_slabs`` issues it: eagerly, for the
count read once on the host; under stream capture, as the bodies of one SWITCH conditional graph
node whose value a captured kernel sets from the device-side count when the graph runs
(``vb_slab_switch`` / ``vb_slab_begin`` / ``vb_slab_close``), so the captured train step stays one
graph whose replays follow the live active count with one launch per operation. Bodies allocate
nothing: cuBLAS GEMMs and this library's kernels write into buffers allocated before the switch.

``slab_ffn`` is the feed-forward block ``W_2 relu(W_1 x)^2`` (``vesper/ffn.py:20-60``) on a compact
buffer, forward and backward.
"""

from __future__ import annotations

import ctypes
from collections.abc import Callable

import torch
from torch import Tensor

from vesper_b200 import _lib

SLAB_FIRST = 1024  # rows of the smallest bucket (the buckets double from there)

_SIDE: dict[int, torch.cuda.Stream] = {}


def bucket_ends(cap: int, first: int = SLAB_FIRST) -> list[int]:
    """``[first, 2 first, 4 first, ..., cap]``: the ends of the buckets ``[0, end)`` (the
    numbering ``vb_slab_switch`` uses)."""
    ends: list[int] = []
    end = min(first, cap)
    while cap > 0:
        ends.append(end)
        if end >= cap:
            break
        end = min(2 * end, cap)
    return ends


def bucket_end(count: int, cap: int, first: int = SLAB_FIRST) -> int:
    """The end of the bucket that runs for ``count`` active rows (0 for none)."""
    return 0 if count <= 0 else next(e for e in bucket_ends(cap, first) if e >= min(count, cap))


def body_stream(device: torch.device) -> torch.cuda.Stream:
    """The stream the bucket bodies are issued on (one per device, kept: cuBLAS's workspace for it
    is allocated by the first, eager use, never inside a capture)."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    stream = _SIDE.get(index)
    if stream is None:
        stream = torch.cuda.Stream(device=torch.device("cuda", index))
        _SIDE[index] = stream
    return stream


def run_slabs(count: Tensor, cap: int, body: Callable[[int], None], first: int = SLAB_FIRST) -> None:
    """Issue ``body(end)``, the work over rows ``[0, end)``, for the bucket that holds ``count``
    (int32 ``[1]`` on the device) active rows, nothing for none. ``body`` runs on the bucket
    stream with autocast off and must not allocate device memory."""
    if cap <= 0:
        return
    ends = bucket_ends(cap, first)
    main = torch.cuda.current_stream(count.device)
    side = body_stream(count.device)
    if torch.cuda.is_current_stream_capturing():
        bodies = (ctypes.c_void_p * len(ends))()
        _lib.call("vb_slab_switch", count.data_ptr(), cap, first, main.cuda_stream, bodies)
        for graph, end in zip(bodies, ends, strict=True):
            _lib.call("vb_slab_begin", graph, side.cuda_stream)
            try:
                with torch.cuda.stream(side), torch.autocast("cuda", enabled=False):
                    body(end)
            finally:
                _lib.call("vb_slab_close", side.cuda_stream)
        return
    end = bucket_end(int(count.item()), cap, first)
    if end == 0:
        return
    side.wait_stream(main)
    with torch.cuda.stream(side), torch.autocast("cuda", enabled=False):
        body(end)
    main.wait_stream(side)


class _SlabFFN(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, w1: Tensor, w2: Tensor, count: Tensor, first: int) -> Tensor:  # type: ignore[override]
        cap, hidden = x.shape[0], w1.shape[0]
        h = x.new_empty(cap, hidden)
        g = x.new_empty(cap, hidden)
        y = x.new_empty(cap, w2.shape[0])
        code = _lib.DTYPE_CODE[x.dtype]

        def body(e: int) -> None:
            torch.mm(x[:e], w1.t(), out=h[:e])
            _lib.call("vb_relu_square_fwd", h.data_ptr(), g.data_ptr(), e * hidden, code, _lib.stream(x.device))
            torch.mm(g[:e], w2.t(), out=y[:e])

        run_slabs(count, cap, body, first)
        ctx.save_for_backward(x, w1, w2, h, g, count)
        ctx.first = first
        return y

    @staticmethod
    def backward(ctx, dy: Tensor):  # type: ignore[override]
        x, w1, w2, h, g, count = ctx.saved_tensors
        dy = dy.contiguous().to(x.dtype)
        cap, hidden = x.shape[0], w1.shape[0]
        dg, dh, dx = torch.empty_like(g), torch.empty_like(h), torch.empty_like(x)
        dw1, dw2 = torch.zeros_like(w1), torch.zeros_like(w2)  # what no bucket writes: no active row
        code = _lib.DTYPE_CODE[x.dtype]

        def body(e: int) -> None:
            torch.mm(dy[:e], w2, out=dg[:e])
            torch.mm(dy[:e].t(), g[:e], out=dw2)
            _lib.call("vb_relu_square_bwd", h.data_ptr(), dg.data_ptr(), dh.data_ptr(), e * hidden, code,
                      _lib.stream(x.device))  # fmt: skip
            torch.mm(dh[:e].t(), x[:e], out=dw1)
            torch.mm(dh[:e], w1, out=dx[:e])

        run_slabs(count, cap, body, ctx.first)
        return dx, dw1, dw2, None, None


def slab_ffn(x: Tensor, w1: Tensor, w2: Tensor, count: Tensor, first: int = SLAB_FIRST) -> Tensor:
    """``W_2 relu(W_1 x)^2`` over the first ``count`` rows of the compact buffer ``x [cap, d]``
    (bucketed work; the rows from the count to the end of its bucket must be finite, as
    ``gather_rows`` over a ``compact_flat`` compaction leaves them). ``w1 [hidden, d]``,
    ``w2 [d, hidden]`` in ``x``'s dtype. Rows past the bucket of the result are undefined; the
    weights' gradients are zero when no row is active."""
    return _SlabFFN.apply(x.contiguous(), w1.contiguous(), w2.contiguous(), count, first)
