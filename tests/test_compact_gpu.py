"""The loop's compaction and row-copy kernels on a B200, bit for bit against torch indexing.

Byte work, so the bar is equality: the index list, ranks and counts of ``compact_index`` against
``nonzero``; ``select_rows`` against ``torch.where`` (the reference's ``_carry`` / ``_merge``,
vesper/column.py:140-143 and vesper/loop.py:523-537) for every dtype and row width the loop
carries, odd widths included; gather/expand round trips; and every backward against the
gradient of the torch expression.
"""

from __future__ import annotations

import pytest
import torch

from vesper_b200.kernels.compact import compact_flat, compact_index, expand_rows, gather_rows, select_rows
from vesper_b200.kernels.slabs import bucket_end

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")


def _active(b: int, n: int, p: float, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    return (torch.rand(b, n, generator=g) < p).to(CUDA)


@pytest.mark.parametrize(("b", "n", "p"), [(3, 1, 0.5), (2, 1000, 0.3), (4, 2048, 0.9), (2, 3000, 0.0), (1, 5000, 1.0)])
def test_compact_index_matches_nonzero(b: int, n: int, p: float) -> None:
    active = _active(b, n, p, seed=n)
    comp = compact_index(active, qpos_offset=17)
    for i in range(b):
        idx = active[i].nonzero().flatten().to(torch.int32)
        c = idx.numel()
        assert int(comp.counts[i]) == c
        assert torch.equal(comp.idx[i, :c], idx)
        assert torch.equal(comp.qpos[i, :c], idx + 17)
        assert bool((comp.idx[i, c:] == -1).all())
        rank = torch.full((n,), -1, dtype=torch.int32, device=CUDA)
        rank[idx.long()] = torch.arange(c, dtype=torch.int32, device=CUDA)
        assert torch.equal(comp.rank[i], rank)


def _tensors(b: int, n: int, seed: int) -> list[torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    shapes = [((b, n, 64), torch.bfloat16), ((b, n, 2, 32), torch.float32), ((b, n, 2), torch.bfloat16),
              ((b, n, 3), torch.float32), ((b, n, 5), torch.float16), ((b, n, 1, 64), torch.bfloat16)]  # fmt: skip
    return [torch.randn(*s, generator=g).to(dt).to(CUDA) for s, dt in shapes]


def test_select_rows_equals_where_forward_and_backward() -> None:
    b, n = 3, 333
    active = _active(b, n, 0.6, seed=1)
    fresh = [t.requires_grad_() for t in _tensors(b, n, 2)]
    carried = [t.requires_grad_() for t in _tensors(b, n, 3)]
    out = select_rows(active, fresh, carried)
    want = [torch.where(active.reshape(b, n, *[1] * (f.dim() - 2)), f, c) for f, c in zip(fresh, carried, strict=True)]
    assert all(torch.equal(a, w) for a, w in zip(out, want, strict=True))
    ups = [torch.randn_like(o) for o in out]
    got_g = torch.autograd.grad([(o.float() * u.float()).sum() for o, u in zip(out, ups, strict=True)], fresh + carried)
    want_g = torch.autograd.grad([(w.float() * u.float()).sum() for w, u in zip(want, ups, strict=True)], fresh + carried)
    assert all(torch.equal(a, w) for a, w in zip(got_g, want_g, strict=True))


def test_select_rows_with_zero_fallback() -> None:
    active = _active(2, 100, 0.5, seed=4)
    (x,) = _tensors(2, 100, 5)[:1]
    (out,) = select_rows(active, [x], [None])
    assert torch.equal(out, torch.where(active[..., None], x, torch.zeros_like(x)))


def test_gather_then_expand_round_trips_and_backward_is_exact() -> None:
    b, n = 2, 700
    active = _active(b, n, 0.4, seed=6)
    comp = compact_index(active)
    dense = [t.requires_grad_() for t in _tensors(b, n, 7)]
    packed = gather_rows(comp, dense)
    for d, p in zip(dense, packed, strict=True):
        for i in range(b):
            c = int(comp.counts[i])
            assert torch.equal(p[i, :c], d[i][active[i]])
            assert not p[i, c:].any()
    fallback = _tensors(b, n, 8)
    back = expand_rows(comp, packed, fallback)
    for d, f, r in zip(dense, fallback, back, strict=True):
        assert torch.equal(r, torch.where(active.reshape(b, n, *[1] * (d.dim() - 2)), d, f))
    ups = [torch.randn_like(r) for r in back]
    grads = torch.autograd.grad([(r.float() * u.float()).sum() for r, u in zip(back, ups, strict=True)], dense)
    for gd, u in zip(grads, ups, strict=True):
        assert torch.equal(gd, torch.where(active.reshape(b, n, *[1] * (u.dim() - 2)), u, torch.zeros_like(u)))


def test_empty_batches_and_capture() -> None:
    active = torch.zeros(2, 64, dtype=torch.bool, device=CUDA)
    comp = compact_index(active)
    assert comp.counts.tolist() == [0, 0]
    x = torch.randn(2, 64, 16, device=CUDA)
    graph = torch.cuda.CUDAGraph()
    act = _active(2, 64, 0.5, seed=9)
    with torch.cuda.graph(graph):
        c2 = compact_index(act)
        (pk,) = gather_rows(c2, [x])
        (bk,) = expand_rows(c2, [pk])
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(bk, torch.where(act[..., None], x, torch.zeros_like(x)))


@pytest.mark.parametrize(("b", "n", "p"), [(3, 700, 0.3), (4, 2048, 0.05), (2, 1000, 0.0), (2, 1500, 1.0)])
def test_the_flat_compaction_and_its_relayout_match_nonzero(b: int, n: int, p: float) -> None:
    """``compact_flat``: every active token of the batch in row order, its rank, the total, and
    the maps between flat compact rows and the per-row compact rows ``(b, r)`` at ``b n + r``."""
    active = _active(b, n, p, seed=b * n)
    rows = compact_flat(active, 256)
    flat = active.reshape(-1).nonzero().flatten().to(torch.int32)
    c = flat.numel()
    assert int(rows.counts[0]) == c
    assert torch.equal(rows.idx[0, :c], flat)
    rank = torch.full((b * n,), -1, dtype=torch.int32, device=CUDA)
    rank[flat.long()] = torch.arange(c, dtype=torch.int32, device=CUDA)
    assert torch.equal(rows.rank[0], rank)
    counts = active.sum(1).tolist()
    per_row = [b_ * n + r for b_ in range(b) for r in range(counts[b_])]
    assert rows.relayout is not None
    assert rows.relayout.idx[0, :c].tolist() == per_row
    pb = torch.full((b * n,), -1, dtype=torch.int32)
    pb[torch.tensor(per_row, dtype=torch.long)] = torch.arange(c, dtype=torch.int32)
    assert torch.equal(rows.relayout.rank[0].cpu(), pb)


def test_the_bucketed_gather_zeroes_to_the_bucket_end_and_leaves_the_rest() -> None:
    """Rows from the count to the end of the count's bucket are zero; rows past it keep what the
    buffer held (nothing reads them); the expand back restores the active rows exactly."""
    b, n, d, first = 2, 3000, 48, 256
    active = _active(b, n, 0.05, seed=9)
    rows = compact_flat(active, first)
    x = torch.randn(1, b * n, d, device=CUDA)
    (xc,) = gather_rows(rows, [x])
    c = int(rows.counts[0])
    end = bucket_end(c, b * n, first)
    assert end >= c and end < b * n
    assert torch.equal(xc[0, :c], x[0, rows.idx[0, :c].long()])
    assert bool((xc[0, c:end] == 0).all())
    (back,) = expand_rows(rows, [xc])
    keep = active.reshape(1, -1, 1)
    assert torch.equal(torch.where(keep, back, 0.0), torch.where(keep, x, 0.0))
    assert bool((back[~keep.expand_as(back)] == 0).all())
