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
    def forward(ctx, x: Tensor, w1: Tensor, w2: Tensor, count: Tensor, first: int,  # type: ignore[override]
                base: Tensor | None) -> Tensor:  # fmt: skip
        cap, hidden = x.shape[0], w1.shape[0]
        h = x.new_empty(cap, hidden)
        g = x.new_empty(cap, hidden)
        y = x.new_empty(cap, w2.shape[0])
        out = torch.empty_like(base) if base is not None else y
        code = _lib.DTYPE_CODE[x.dtype]

        def body(e: int) -> None:
            torch.mm(x[:e], w1.t(), out=h[:e])
            _lib.call("vb_relu_square_fwd", h.data_ptr(), g.data_ptr(), e * hidden, code, _lib.stream(x.device))
            torch.mm(g[:e], w2.t(), out=y[:e])
            if base is not None:  # the residual: base + y in float32, one rounding-free add
                _lib.call("vb_residual_add", base.data_ptr(), y.data_ptr(), None, out.data_ptr(), e, base.shape[1],
                          code, _lib.stream(x.device))  # fmt: skip

        run_slabs(count, cap, body, first)
        ctx.save_for_backward(x, w1, w2, h, g, count)
        ctx.first, ctx.residual = first, base is not None
        return out

    @staticmethod
    def backward(ctx, dout: Tensor):  # type: ignore[override]
        x, w1, w2, h, g, count = ctx.saved_tensors
        dout = dout.contiguous()
        cap, hidden = x.shape[0], w1.shape[0]
        dy = torch.empty(cap, w2.shape[0], dtype=x.dtype, device=x.device) if ctx.residual else dout.to(x.dtype)
        dg, dh, dx = torch.empty_like(g), torch.empty_like(h), torch.empty_like(x)
        dw1, dw2 = torch.zeros_like(w1), torch.zeros_like(w2)  # what no bucket writes: no active row
        code = _lib.DTYPE_CODE[x.dtype]

        def body(e: int) -> None:
            if ctx.residual:  # y's gradient: the output's, rounded to y's dtype
                _lib.call("vb_residual_add_bwd", dout.data_ptr(), None, None, dy.data_ptr(), e, dout.shape[1], code,
                          _lib.stream(x.device))  # fmt: skip
            torch.mm(dy[:e], w2, out=dg[:e])
            torch.mm(dy[:e].t(), g[:e], out=dw2)
            _lib.call("vb_relu_square_bwd", h.data_ptr(), dg.data_ptr(), dh.data_ptr(), e * hidden, code,
                      _lib.stream(x.device))  # fmt: skip
            torch.mm(dh[:e].t(), x[:e], out=dw1)
            torch.mm(dh[:e], w1, out=dx[:e])

        run_slabs(count, cap, body, ctx.first)
        return dx, dw1, dw2, None, None, (dout if ctx.residual else None)


def slab_ffn(x: Tensor, w1: Tensor, w2: Tensor, count: Tensor, first: int = SLAB_FIRST,
             residual: Tensor | None = None) -> Tensor:  # fmt: skip
    """``W_2 relu(W_1 x)^2`` over the first ``count`` rows of the compact buffer ``x [cap, d]``
    (bucketed work; the rows from the count to the end of its bucket must be finite, as
    ``gather_rows`` over a ``compact_flat`` compaction leaves them). ``w1 [hidden, d]``,
    ``w2 [d, hidden]`` in ``x``'s dtype. With ``residual`` (float32 ``[cap, d]``) the result is
    ``residual + W_2 relu(W_1 x)^2`` in float32 (the column's last residual add). Rows past the
    bucket of the result are undefined; the weights' gradients are zero when no row is active."""
    base = None if residual is None else residual.contiguous()
    return _SlabFFN.apply(x.contiguous(), w1.contiguous(), w2.contiguous(), count, first, base)


class _SlabResidualNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, o: Tensor, gain: Tensor, count: Tensor, first: int, floor: float, eps: float,  # type: ignore[override]
                w: Tensor) -> tuple[Tensor, Tensor]:  # fmt: skip
        cap, d = x.shape
        r = o.new_empty(cap, d, dtype=w.dtype)
        s = torch.empty_like(x)
        y = x.new_empty(cap, d, dtype=w.dtype)
        inv = x.new_empty(cap, dtype=torch.float32)
        g32 = gain.to(torch.float32).contiguous()

        def body(e: int) -> None:
            torch.mm(o[:e], w.t(), out=r[:e])
            _lib.call(
                "vb_add_rms_norm_fwd", x.data_ptr(), r.data_ptr(), g32.data_ptr(), s.data_ptr(), y.data_ptr(),
                inv.data_ptr(), e, d, floor, eps, _lib.DTYPE_CODE[r.dtype], _lib.DTYPE_CODE[y.dtype],
                _lib.stream(x.device),
            )  # fmt: skip

        run_slabs(count, cap, body, first)
        ctx.save_for_backward(o, w, s, g32, inv, count)
        ctx.first, ctx.gain_dtype = first, gain.dtype
        return s, y

    @staticmethod
    def backward(ctx, ds: Tensor | None, dy: Tensor | None):  # type: ignore[override]
        o, w, s, g32, inv, count = ctx.saved_tensors
        cap, d = s.shape
        dy = torch.zeros(cap, d, dtype=w.dtype, device=s.device) if dy is None else dy.contiguous().to(w.dtype)
        ds = None if ds is None else ds.contiguous().to(torch.float32)
        dx = torch.empty_like(s)
        dr = torch.empty(cap, d, dtype=w.dtype, device=s.device)
        do = torch.empty_like(o)
        dw = torch.zeros_like(w)  # what no bucket writes: no active row
        dg = torch.zeros(d, dtype=torch.float32, device=s.device)
        ws = _lib.workspace(_lib.query("vb_rms_norm_bwd_workspace", cap, d), s.device)

        def body(e: int) -> None:
            _lib.call(
                "vb_add_rms_norm_bwd", s.data_ptr(), g32.data_ptr(), dy.data_ptr(), inv.data_ptr(), _lib.ptr(ds),
                dx.data_ptr(), dr.data_ptr(), dg.data_ptr(), ws.data_ptr(), e, d, _lib.DTYPE_CODE[dy.dtype],
                _lib.DTYPE_CODE[dr.dtype], _lib.stream(s.device),
            )  # fmt: skip
            torch.mm(dr[:e], w, out=do[:e])
            torch.mm(dr[:e].t(), o[:e], out=dw)

        run_slabs(count, cap, body, ctx.first)
        return dx, do, dg.to(ctx.gain_dtype), None, None, None, None, dw


def slab_residual_norm(x: Tensor, o: Tensor, w: Tensor, gain: Tensor, count: Tensor, first: int = SLAB_FIRST,
                       floor: float = 1e-3, eps: float = 1e-6) -> tuple[Tensor, Tensor]:  # fmt: skip
    """``(s, y)`` over the first ``count`` rows of compact buffers: the residual add
    ``s = x + o W^T`` (float32 ``x``; the product in ``w``'s dtype, added as one float32 addition)
    and the RMSNorm of the sum rounded to ``w``'s dtype (``vb_add_rms_norm_fwd``: a sublayer's
    output projection, its residual add and the next sublayer's norm). Width a multiple of 4 up to
    1024. Rows past the bucket are undefined; ``w``'s and the gain's gradients are zero when no
    row is active."""
    return _SlabResidualNorm.apply(x.contiguous(), o.contiguous(), gain, count, first, floor, eps, w.contiguous())


class _SlabLinears(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: Tensor, gain: Tensor | None, count: Tensor, first: int, floor: float, eps: float,  # type: ignore[override]
                pos: Tensor | None, freq: Tensor | None, turns: tuple[int, ...], *weights: Tensor) -> tuple[Tensor, ...]:  # fmt: skip
        cap, d = x.shape
        dtype = weights[0].dtype
        norm = gain is not None
        xn = x.new_empty(cap, d, dtype=dtype) if norm else x
        inv = x.new_empty(cap, dtype=torch.float32) if norm else None
        g32 = gain.to(torch.float32).contiguous() if gain is not None else None
        outs = [x.new_empty(cap, w.shape[0], dtype=dtype) for w in weights]
        raws = [x.new_empty(cap, w.shape[0], dtype=dtype) if h else None for w, h in zip(weights, turns, strict=True)]

        def body(e: int) -> None:
            if norm:
                _lib.call(
                    "vb_rms_norm_fwd_cast", x.data_ptr(), g32.data_ptr(), xn.data_ptr(), inv.data_ptr(), e, d,
                    floor, eps, _lib.DTYPE_CODE[x.dtype], _lib.DTYPE_CODE[dtype], _lib.stream(x.device),
                )  # fmt: skip
            for w, o, raw, heads in zip(weights, outs, raws, turns, strict=True):
                if raw is None:
                    torch.mm(xn[:e], w.t(), out=o[:e])
                    continue
                torch.mm(xn[:e], w.t(), out=raw[:e])
                _rotate(raw, pos, freq, o, e, heads, backward=False)

        run_slabs(count, cap, body, first)
        ctx.save_for_backward(x, g32, xn, inv, count, pos, freq, *weights)
        ctx.first, ctx.norm, ctx.turns = first, norm, turns
        ctx.gain_dtype = None if gain is None else gain.dtype
        return tuple(outs)

    @staticmethod
    def backward(ctx, *douts: Tensor | None):  # type: ignore[override]
        x, g32, xn, inv, count, pos, freq, *weights = ctx.saved_tensors
        cap, d = x.shape
        grads = [None if g is None else g.contiguous().to(xn.dtype) for g in douts]
        unturned = [torch.empty_like(g) if g is not None and h else None for g, h in zip(grads, ctx.turns, strict=True)]
        dxn = torch.empty_like(xn)
        dws = [torch.zeros_like(w) for w in weights]  # what no bucket writes: no active row
        dx = torch.empty_like(x) if ctx.norm else dxn
        dg = torch.zeros(d, dtype=torch.float32, device=x.device) if ctx.norm else None
        ws = _lib.workspace(_lib.query("vb_rms_norm_bwd_workspace", cap, d), x.device) if ctx.norm else None

        def body(e: int) -> None:
            started = False
            for w, g, gu, dw, heads in zip(weights, grads, unturned, dws, ctx.turns, strict=True):
                if g is None:
                    continue
                if gu is not None:  # the rotation's transpose first
                    _rotate(g, pos, freq, gu, e, heads, backward=True)
                    g = gu
                if started:
                    dxn[:e].addmm_(g[:e], w)  # accumulated in the product's epilogue, no separate add
                else:
                    torch.mm(g[:e], w, out=dxn[:e])
                    started = True
                torch.mm(g[:e].t(), xn[:e], out=dw)
            if not started:
                dxn[:e].zero_()
            if ctx.norm:
                _lib.call(
                    "vb_rms_norm_bwd_cast", x.data_ptr(), g32.data_ptr(), dxn.data_ptr(), inv.data_ptr(),
                    dx.data_ptr(), dg.data_ptr(), ws.data_ptr(), e, d, _lib.DTYPE_CODE[x.dtype],
                    _lib.DTYPE_CODE[dxn.dtype], _lib.stream(x.device),
                )  # fmt: skip

        run_slabs(count, cap, body, ctx.first)
        dgain = None if dg is None else dg.to(ctx.gain_dtype)
        return (dx, dgain, None, None, None, None, None, None, None, *dws)


def _rotate(src: Tensor, pos: Tensor, freq: Tensor, dst: Tensor, rows: int, heads: int, *, backward: bool) -> None:
    """The rotary turn of rows ``[0, rows)`` of ``src [cap, heads * dk]`` into ``dst``
    (``vb_rotary``; ``backward``: the transposed turn of a gradient)."""
    dk = src.shape[1] // heads
    _lib.call(
        "vb_rotary", src.data_ptr(), pos.data_ptr(), freq.data_ptr(), dst.data_ptr(), rows, heads, dk, int(backward),
        _lib.DTYPE_CODE[src.dtype], _lib.stream(src.device),
    )  # fmt: skip


def slab_linears(x: Tensor, weights: list[Tensor], count: Tensor, first: int = SLAB_FIRST,
                 norm: tuple[Tensor, float, float] | None = None,
                 rotary: tuple[Tensor, Tensor, tuple[int, ...]] | None = None) -> tuple[Tensor, ...]:  # fmt: skip
    """``[x_n W^T for W in weights]`` over the first ``count`` rows of the compact buffer
    ``x [cap, d]`` (bucketed work, the rows up to the bucket's end finite), ``x_n = x`` or, with
    ``norm = (gain, floor, eps)``, the RMSNorm of a float32 ``x`` rounded to the weights' dtype
    (``vb_rms_norm_fwd_cast``: the column's norm followed by its projections). ``rotary = (pos
    int64 [cap], inv_freq float64 [dk/2], heads per output)`` turns each output with a nonzero
    head count by the rotary embedding at its row's position (``vb_rotary``; 0: not turned). The
    backward forms ``x_n``'s gradient as one accumulated product chain (no separate adds). Rows
    past the bucket of the results are undefined; the weights' and gain's gradients are zero when
    no row is active."""
    gain, floor, eps = norm if norm is not None else (None, 0.0, 0.0)
    if norm is None and x.dtype != weights[0].dtype:
        msg = f"x ({x.dtype}) and the weights ({weights[0].dtype}) must share a dtype without a norm"
        raise ValueError(msg)
    pos, freq, turns = rotary if rotary is not None else (None, None, (0,) * len(weights))
    if len(turns) != len(weights):
        msg = f"rotary: {len(turns)} head counts for {len(weights)} weights"
        raise ValueError(msg)
    return _SlabLinears.apply(x.contiguous(), gain, count, first, floor, eps, pos, freq, tuple(turns),
                              *[w.contiguous() for w in weights])  # fmt: skip
