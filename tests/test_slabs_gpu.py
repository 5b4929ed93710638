"""Slab-sized work over a device-side count (``vesper_b200.kernels.slabs``): the feed-forward block
on the active rows only, eager and inside a captured graph whose replays follow the live count.

The reference runs the block over every token and discards the halted rows (``vesper/loop.py:
24-26``); the compact form must give the same values at the active rows, zero at the others, and
the same gradients (the halted rows contribute nothing to the weights' gradients because the loop
zeroes their outputs).
"""

from __future__ import annotations

import pytest
import torch

from conftest import elem_rel, max_rel, rel
from vesper_b200 import _lib
from vesper_b200.kernels.compact import compact_flat, expand_rows, gather_rows
from vesper_b200.kernels.slabs import bucket_end, bucket_ends, slab_ffn, slab_linears

FIRST = 512


def _dense(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, active: torch.Tensor) -> torch.Tensor:
    """The reference's block (``vesper/ffn.py:44-56``: relu, then the product in x's dtype) over
    every row, the halted rows' outputs replaced by zero."""
    h = torch.relu(x @ w1.t())
    return torch.where(active[..., None], (h * h) @ w2.t(), 0.0)


def _compact(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, active: torch.Tensor) -> torch.Tensor:
    b, n, d = x.shape
    rows = compact_flat(active, FIRST)
    (xc,) = gather_rows(rows, [x.reshape(1, b * n, d)])
    yc = slab_ffn(xc[0], w1, w2, rows.counts, FIRST)
    (y,) = expand_rows(rows, [yc.view(1, b * n, -1)])
    return y.view(b, n, -1)


def _inputs(dtype: torch.dtype, frac: float, seed: int) -> tuple[torch.Tensor, ...]:
    g = torch.Generator(device="cuda").manual_seed(seed)
    b, n, d, hidden = 4, 1536, 64, 192  # 6144 rows: buckets [0, 512), [0, 1024), ... [0, 6144)
    x = torch.randn(b, n, d, device="cuda", generator=g).to(dtype)
    w1 = (torch.randn(hidden, d, device="cuda", generator=g) / d**0.5).to(dtype)
    w2 = (torch.randn(d, hidden, device="cuda", generator=g) / hidden**0.5).to(dtype)
    active = torch.rand(b, n, device="cuda", generator=g) < frac
    up = torch.randn(b, n, d, device="cuda", generator=g).to(dtype)
    return x, w1, w2, active, up


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("frac", [0.0, 0.0005, 0.07, 0.4, 1.0])
def test_the_compact_block_matches_the_dense_one_at_the_active_rows(dtype: torch.dtype, frac: float) -> None:
    x, w1, w2, active, up = _inputs(dtype, frac, 7)
    leaves = [t.detach().requires_grad_() for t in (x, w1, w2)]
    y = _compact(*leaves, active)
    grads = torch.autograd.grad([(y.float() * up.float()).sum()], leaves)
    ref_leaves = [t.detach().double().requires_grad_() for t in (x, w1, w2)]
    y_ref = _dense(*ref_leaves, active)
    ref_grads = torch.autograd.grad([(y_ref * up.double()).sum()], ref_leaves)
    assert torch.all(y[~active] == 0)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    for got, want in [(y, y_ref), *zip(grads, ref_grads, strict=True)]:
        got_np, want_np = got.detach().double().cpu().numpy(), want.detach().cpu().numpy()
        if not want_np.any():
            assert not got_np.any()
            continue
        assert max_rel(got_np, want_np) < tol
        assert rel(got_np, want_np) < tol
        if dtype == torch.float32:
            assert elem_rel(got_np, want_np) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("frac", [0.0, 0.003, 0.3, 1.0])
def test_the_compact_norm_and_projections_match_the_dense_ones(dtype: torch.dtype, frac: float) -> None:
    """``slab_linears`` with the norm (float32 rows, the RMSNorm rounded to ``dtype``, four
    projections) against the reference's norm and linears at the active rows."""
    g = torch.Generator(device="cuda").manual_seed(5)
    b, n, d, heads = 2, 1536, 64, 4
    x = torch.randn(b, n, d, device="cuda", generator=g) * 3
    gain = 1 + 0.1 * torch.randn(d, device="cuda", generator=g)
    ws = [torch.randn(o, d, device="cuda", generator=g) / d**0.5 for o in (d, d, d, heads)]
    active = torch.rand(b, n, device="cuda", generator=g) < frac
    ups = [torch.randn(b, n, w.shape[0], device="cuda", generator=g) for w in ws]
    leaves = [t.detach().requires_grad_() for t in (x, gain, *ws)]
    rows = compact_flat(active, FIRST)
    (xc,) = gather_rows(rows, [leaves[0].reshape(1, b * n, d)])
    outs = slab_linears(xc[0], [w.to(dtype) for w in leaves[2:]], rows.counts, FIRST, norm=(leaves[1], 1e-3, 1e-6))
    dense = expand_rows(rows, [o.view(1, b * n, -1) for o in outs])
    loss = sum((y.float().view(b, n, -1) * u).sum() for y, u in zip(dense, ups, strict=True))
    grads = torch.autograd.grad([loss], leaves)

    ref = [t.detach().double().requires_grad_() for t in (x, gain, *ws)]
    xr, gr = ref[0], ref[1]
    xn = xr * torch.rsqrt(xr.square().mean(-1, keepdim=True) + 1e-6) * gr  # vesper/column.py:159-188, exact
    ref_outs = [torch.where(active[..., None], xn @ w.t(), 0.0) for w in ref[2:]]
    ref_loss = sum((y * u.double()).sum() for y, u in zip(ref_outs, ups, strict=True))
    ref_grads = torch.autograd.grad([ref_loss], ref)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    pairs = [(y.view(b, n, -1), r) for y, r in zip(dense, ref_outs, strict=True)]
    for got, want in [*pairs, *zip(grads, ref_grads, strict=True)]:
        got_np, want_np = got.detach().double().cpu().numpy(), want.detach().cpu().numpy()
        if not want_np.any():
            assert not got_np.any()
            continue
        assert max_rel(got_np, want_np) < tol
        assert rel(got_np, want_np) < tol


@pytest.mark.gpu
def test_a_captured_graph_runs_the_slabs_the_live_count_needs() -> None:
    """One capture, replayed under masks of 0, 1, some and all active tokens: bitwise the eager
    results (the bucket the count selects runs the same products in both)."""
    dtype = torch.bfloat16
    x, w1, w2, active, up = _inputs(dtype, 0.1, 11)
    leaves = [t.detach().requires_grad_() for t in (x, w1, w2)]
    static_active = active.clone()

    def step() -> list[torch.Tensor]:
        y = _compact(*leaves, static_active)
        grads = torch.autograd.grad([(y.float() * up.float()).sum()], leaves)
        return [y, *grads]

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = step()
    g = torch.Generator(device="cuda").manual_seed(3)
    b, n = active.shape
    masks = [
        torch.zeros(b, n, dtype=torch.bool, device="cuda"),
        torch.zeros(b, n, dtype=torch.bool, device="cuda").index_fill_(1, torch.tensor([777], device="cuda"), True),
        torch.rand(b, n, device="cuda", generator=g) < 0.05,
        torch.rand(b, n, device="cuda", generator=g) < 0.6,
        torch.ones(b, n, dtype=torch.bool, device="cuda"),
    ]
    for mask in masks:
        static_active.copy_(mask)
        graph.replay()
        torch.cuda.synchronize()
        captured = [t.clone() for t in outs]
        eager = step()
        for c, e in zip(captured, eager, strict=True):
            assert torch.equal(c, e)
        assert torch.all(captured[0][~mask] == 0)
    del graph


def test_the_bucket_count_of_the_library_matches_the_host_numbering() -> None:
    """Host-only: the library's bucket numbering (no kernel call, runs without a GPU)."""
    for cap in (1, 511, 512, 513, 2048, 6144, 65536, 100_000):
        ends = bucket_ends(cap, FIRST)
        assert _lib.query("vb_slab_count", cap, FIRST) == len(ends)
        assert ends[-1] == cap and all(b == min(2 * a, cap) for a, b in zip(ends, ends[1:], strict=False))
    assert bucket_end(0, 6144, FIRST) == 0
    assert bucket_end(1, 6144, FIRST) == 512
    assert bucket_end(513, 6144, FIRST) == 1024
    assert bucket_end(4097, 6144, FIRST) == 6144
