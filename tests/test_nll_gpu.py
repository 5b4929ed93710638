"""``linear_nll`` (the head's fused per-token loss) on a B200 against torch's cross-entropy.

The oracle is torch's own ``cross_entropy`` over ``F.linear(x, weight)`` (the path the reference's
``linear_nll`` replaced, ``vesper/kernels/nll.py:1-40``; its tests ``tests/test_nll.py``): in
float32 the losses and both gradients agree to float32 rounding; under bf16 autocast (the same
rounding points: bf16 logits, float32 softmax, the logits' gradient in bf16 before the matmuls)
to bf16 rounding. A common offset of a row's logits cancels, kept and recomputed logits give the
same results, a captured call equals the eager one bitwise, and bad targets are refused.
"""

from __future__ import annotations

import pytest
import torch
from torch.nn import functional

from conftest import rel
from vesper_b200 import _lib
from vesper_b200.contracts import ContractError
from vesper_b200.kernels.nll import linear_nll, row_stats

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")


def _inputs(n, d, vocab, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = (torch.randn(n, d, generator=g) * 0.5).to(CUDA)
    w = (torch.randn(vocab, d, generator=g) * 0.05).to(CUDA)
    t = torch.randint(0, vocab, (n,), generator=g).to(CUDA)
    up = torch.rand(n, generator=g).to(CUDA)
    return x, w, t, up


def _grads(fn, x, w, t, up, *, autocast: bool):
    xs, ws = x.clone().requires_grad_(), w.clone().requires_grad_()
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
        loss = fn(xs, ws, t)
    (loss.float() * up).sum().backward()
    return [loss.detach().double(), xs.grad.double(), ws.grad.double()]


def _oracle(x, w, t):
    logits = functional.linear(x, w)
    return functional.cross_entropy(logits.float(), t, reduction="none")


@pytest.mark.parametrize(("n", "d", "vocab"), [(300, 64, 1000), (1024, 512, 32000), (77, 96, 50257)])
def test_float32_matches_cross_entropy(n: int, d: int, vocab: int) -> None:
    x, w, t, up = _inputs(n, d, vocab)
    got = _grads(linear_nll, x, w, t, up, autocast=False)
    want = _grads(_oracle, x, w, t, up, autocast=False)
    for name, a, b in zip(("loss", "dx", "dw"), got, want, strict=True):
        assert rel(a.cpu().numpy(), b.cpu().numpy()) < 1e-5, (name, rel(a.cpu().numpy(), b.cpu().numpy()))


def test_bf16_autocast_matches_the_autocast_cross_entropy() -> None:
    x, w, t, up = _inputs(2048, 512, 32000, seed=1)
    got = _grads(linear_nll, x, w, t, up, autocast=True)
    want = _grads(_oracle, x, w, t, up, autocast=True)
    for name, a, b in zip(("loss", "dx", "dw"), got, want, strict=True):
        assert rel(a.cpu().numpy(), b.cpu().numpy()) < 1e-2, (name, rel(a.cpu().numpy(), b.cpu().numpy()))


def test_a_common_offset_of_a_rows_logits_cancels() -> None:
    g = torch.Generator(device=CUDA).manual_seed(2)
    logits = torch.randn(64, 4096, device=CUDA, generator=g)
    t = torch.randint(0, 4096, (64,), device=CUDA, generator=g)
    _, _, base = row_stats(logits, t)
    for shift in (1e4, -3e3):
        _, _, moved = row_stats(logits + shift, t)
        # only the float32 representation of the shifted logits differs (half an ulp at |shift|)
        assert (moved - base).abs().max().item() < 4e-3, shift


def test_kept_logits_change_memory_not_results() -> None:
    x, w, t, up = _inputs(500, 128, 3000, seed=3)
    a = _grads(lambda xs, ws, tt: linear_nll(xs, ws, tt, keep_logits=True), x, w, t, up, autocast=True)
    b = _grads(linear_nll, x, w, t, up, autocast=True)
    for p, q in zip(a, b, strict=True):
        assert torch.equal(p, q)


def test_a_captured_call_equals_the_eager_one_bitwise() -> None:
    x, w, t, up = _inputs(512, 256, 8000, seed=4)
    xs, ws = x.clone().requires_grad_(), w.clone().requires_grad_()

    def step():
        xs.grad, ws.grad = None, None
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = linear_nll(xs, ws, t)
        (loss * up).sum().backward()
        return [loss.detach().clone(), xs.grad.clone(), ws.grad.clone()]

    eager = step()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    xs.grad, ws.grad = None, None
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            loss = linear_nll(xs, ws, t)
        (loss * up).sum().backward()
        out = [loss, xs.grad, ws.grad]
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        assert all(torch.equal(a, b) for a, b in zip(out, eager, strict=True))
    _lib.check_status(CUDA)


def test_targets_outside_the_vocabulary_and_wrong_shapes_are_refused() -> None:
    x, w, t, _ = _inputs(16, 32, 100, seed=5)
    with pytest.raises(ContractError, match="vocab"):
        linear_nll(x, w, torch.full_like(t, 100))
    with pytest.raises(ContractError, match="axis"):
        linear_nll(x, w[:, :16], t)
    with pytest.raises(ContractError, match="CUDA only"):
        linear_nll(x.cpu(), w.cpu(), t.cpu())
