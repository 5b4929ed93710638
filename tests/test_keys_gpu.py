"""``fused_keys`` on a B200 against the reference's own results (golden vectors) and the oracle.

Bounds follow the reference's kernel test (vesper tests/test_keys_fused.py:58-75): float32 within
2e-5, bfloat16 within 8e-3 (the key's own final rounding), for chunks shorter than the filter
too; the taps' gradient is deterministic (captured == eager, bit for bit).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import golden, golden_names
from vesper_b200.kernels.keys import KEY_NORM_FLOOR, fused_keys, keys_backward, keys_forward

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")


def _run(z, hist, taps, heads, up, want_hist=True):
    zs = z.clone().requires_grad_()
    hs = hist.clone().requires_grad_(want_hist)
    ts = taps.clone().requires_grad_()
    k = fused_keys(zs, hs, ts, heads)
    (k.double() * up.double()).sum().backward()
    return k.detach(), zs.grad, ts.grad, hs.grad


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("name", golden_names("keys_"))
def test_the_fused_keys_equal_the_reference(name: str, dtype: torch.dtype) -> None:
    f = golden(name)
    heads = int(f["heads"])
    z = torch.from_numpy(f["z"]).to(CUDA, dtype)
    hist, taps = (torch.from_numpy(f[k]).to(CUDA, torch.float32) for k in ("hist", "taps"))
    up = torch.from_numpy(f["up"]).to(CUDA)
    k, dz, dtaps, dhist = _run(z, hist, taps, heads, up)
    assert k.dtype == dtype
    bound = 2e-5 if dtype == torch.float32 else 8e-3
    for got, key in ((k, "k"), (dz, "dz"), (dtaps, "dtaps"), (dhist, "dhist")):
        want = f[key]
        got = got.double().cpu().numpy().reshape(want.shape)
        if dtype == torch.float32 or key in ("k", "dhist"):
            np.testing.assert_allclose(got, want, rtol=bound, atol=bound, err_msg=key)
        else:  # bf16 gradients: the upstream gradient and dz are rounded to bf16
            np.testing.assert_allclose(got, want, rtol=2e-2, atol=2e-2 * np.abs(want).max(), err_msg=key)


@pytest.mark.parametrize(("b", "n", "width", "heads"), [(2, 300, 1024, 8), (1, 5, 64, 4), (3, 129, 256, 1)])
def test_wider_shapes_equal_the_oracle(b: int, n: int, width: int, heads: int) -> None:
    g = torch.Generator().manual_seed(n)
    z = torch.randn(b, n, width, generator=g)
    hist = torch.randn(b, 3, width, generator=g)
    taps = torch.randn(4, width, generator=g) * 0.5
    up = torch.randn(b, n, heads, width // heads, generator=g)
    k, dz, dtaps, dhist = _run(z.to(CUDA), hist.to(CUDA), taps.to(CUDA), heads, up.to(CUDA))
    want = oracle.keys(z.numpy(), hist.numpy(), taps.numpy(), heads)
    dz_w, dh_w, dt_w = oracle.keys_grads(z.numpy(), hist.numpy(), taps.numpy(), heads, up.numpy())
    for got, w in ((k, want), (dz, dz_w), (dtaps, dt_w), (dhist, dh_w)):
        np.testing.assert_allclose(got.double().cpu().numpy().reshape(w.shape), w, rtol=2e-5, atol=2e-5)


def test_no_history_gradient_unless_asked_and_captured_equals_eager() -> None:
    g = torch.Generator().manual_seed(3)
    z = torch.randn(2, 64, 128, generator=g).to(CUDA)
    hist = torch.randn(2, 3, 128, generator=g).to(CUDA)
    taps = torch.randn(4, 128, generator=g).to(CUDA)
    up = torch.randn(2, 64, 2, 64, generator=g).to(CUDA)
    _, _, _, dh = _run(z, hist, taps, 2, up, want_hist=False)
    assert dh is None

    def step():
        zs = z.detach().requires_grad_()
        ts = taps.detach().requires_grad_()
        key = fused_keys(zs, hist, ts, 2)
        (key * up).sum().backward()
        return [key.detach().clone(), zs.grad.clone(), ts.grad.clone()]

    eager = [step() for _ in range(2)]
    assert all(torch.equal(a, b) for a, b in zip(eager[0], eager[1], strict=True))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert all(torch.equal(a, b) for a, b in zip(out, eager[0], strict=True))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_saved_statistics_give_the_recomputed_gradients_at_the_clamp_boundary(dtype: torch.dtype) -> None:
    """The backward fed the forward's per-token statistics matches the one that recomputes them,
    also where a head's filtered key is one-hot (squared norm exactly one, gradient through)."""
    g = torch.Generator().manual_seed(11)
    b, n, width, heads, count = 2, 150, 256, 2, 4
    z = torch.randn(b, n, width, generator=g)
    z[0, 10:14, :128] = 0.0
    z[0, 13, 5] = 3.0  # u[0, 13] of head 0 = taps[0, 5] * 3 at channel 5 only
    hist = torch.randn(b, count - 1, width, generator=g).to(CUDA)
    taps = (torch.randn(count, width, generator=g) * 0.5).to(CUDA)
    # u[1, 33] of head 0 has norm 3e-7 at channel 7, below the floor: the clamp holds the gradient
    z[1, 30:34, :128] = 0.0
    z[1, 33, 7] = 3e-7 / float(taps[0, 7])
    zc = z.to(CUDA, dtype)
    grad_k = torch.randn(b, n, heads, width // heads, generator=g).to(CUDA, dtype)
    stats = torch.empty(b, heads, n, 2, device=CUDA)
    keys_forward(zc, hist, taps, heads, KEY_NORM_FLOOR, stats)
    # stats = (r, -1 where the clamp passes gradient): r = 1 / ||u|| above the floor, 1 / floor below
    assert float(stats[0, 0, 13, 1]) == -1.0
    u13 = float(taps[0, 5]) * float(zc[0, 13, 5])
    assert abs(float(stats[0, 0, 13, 0]) * abs(u13) - 1.0) < 1e-6
    assert float(stats[1, 0, 33, 1]) == 1.0
    assert abs(float(stats[1, 0, 33, 0]) * KEY_NORM_FLOOR - 1.0) < 1e-6
    with_stats = keys_backward(zc, hist, taps, grad_k, heads, KEY_NORM_FLOOR, True, stats)
    recomputed = keys_backward(zc, hist, taps, grad_k, heads, KEY_NORM_FLOOR, True, None)
    for got, want in zip(with_stats, recomputed, strict=True):
        w = want.double().cpu().numpy()
        bound = 2e-5 if dtype == torch.float32 else 8e-3
        np.testing.assert_allclose(got.double().cpu().numpy(), w, rtol=bound, atol=bound * np.abs(w).max())

