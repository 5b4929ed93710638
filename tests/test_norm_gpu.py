"""``fused_rms_norm`` on a B200 against the reference's own results and the oracle.

Bounds follow the reference's kernel tests (vesper tests/test_norm_fused.py:48-90): float32 values
and both gradients within 2e-5, bfloat16 activations within 8e-3 (the final rounding); the range
boundaries stay finite; the captured CUDA graph equals the eager call bit for bit and repeats.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import golden, golden_names
from vesper_b200.kernels.norm import fused_rms_norm

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")
FLOOR, EPS = 1e-3, 1e-6


def _run(x: torch.Tensor, gain: torch.Tensor, up: torch.Tensor):
    xs = x.clone().requires_grad_()
    w = gain.clone().requires_grad_()
    y = fused_rms_norm(xs, w, FLOOR, EPS)
    (y.double() * up.double()).sum().backward()
    return y.detach(), xs.grad, w.grad


@pytest.mark.parametrize("name", golden_names("norm_"))
def test_values_and_both_gradients_equal_the_reference(name: str) -> None:
    f = golden(name)
    x, gain, up = (torch.from_numpy(f[k]).to(CUDA) for k in ("x", "gain", "up"))
    y, dx, dg = _run(x, gain, up)
    atol = 1e-6 if name == "norm_boundary" else 2e-5
    np.testing.assert_allclose(y.double().cpu().numpy(), f["y"], rtol=2e-5, atol=atol)
    np.testing.assert_allclose(dx.double().cpu().numpy(), f["dx"], rtol=2e-5, atol=atol)
    if name != "norm_boundary":
        np.testing.assert_allclose(dg.double().cpu().numpy(), f["dg"], rtol=2e-5, atol=2e-5)
    assert torch.isfinite(y).all() and torch.isfinite(dx).all()


@pytest.mark.parametrize("width", [1024, 512, 384, 33, 2048])
def test_bf16_activations_come_back_in_bf16_with_float32_statistics(width: int) -> None:
    g = torch.Generator().manual_seed(width)
    x = (torch.randn(64, width, generator=g) * 50).bfloat16()
    gain = 1 + 0.1 * torch.randn(width, generator=g)
    up = torch.randn(64, width, generator=g)
    y, dx, dg = _run(x.to(CUDA), gain.to(CUDA), up.to(CUDA))
    assert y.dtype == torch.bfloat16 and dx.dtype == torch.bfloat16
    y_want, _ = oracle.rms_norm(x.float().numpy(), gain.numpy())
    dx_want, dg_want = oracle.rms_norm_grads(x.float().numpy(), gain.numpy(), up.bfloat16().float().numpy())
    np.testing.assert_allclose(y.float().cpu().numpy(), y_want, rtol=8e-3, atol=1e-6)
    np.testing.assert_allclose(dx.float().cpu().numpy(), dx_want, rtol=2e-2, atol=2e-3 * np.abs(dx_want).max())
    np.testing.assert_allclose(dg.float().cpu().numpy(), dg_want, rtol=2e-2, atol=1e-2 * np.abs(dg_want).max())


def test_no_rows_give_an_empty_result_and_a_zero_gain_gradient() -> None:
    y, dx, dg = _run(torch.zeros(0, 64, device=CUDA), torch.ones(64, device=CUDA), torch.zeros(0, 64, device=CUDA))
    assert y.shape == (0, 64) and dx.shape == (0, 64)
    assert torch.equal(dg, torch.zeros(64, device=CUDA))


def test_captured_equals_eager_bitwise_and_repeats() -> None:
    x = torch.randn(128, 512, device=CUDA)
    w = torch.ones(512, device=CUDA, requires_grad=True)
    up = torch.randn(128, 512, device=CUDA)

    def step():
        xs = x.detach().requires_grad_()
        w.grad = None
        out = fused_rms_norm(xs, w, FLOOR, EPS)
        (out * up).sum().backward()
        return [out.detach().clone(), xs.grad.clone(), w.grad.clone()]

    eager = [step() for _ in range(2)]
    assert all(torch.equal(a, b) for a, b in zip(eager[0], eager[1], strict=True))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert all(torch.equal(a, b) for a, b in zip(out, eager[0], strict=True))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("width", [512, 1024, 36])
def test_float32_input_rounded_in_the_kernel_equals_the_norm_then_a_cast(dtype: torch.dtype, width: int) -> None:
    """``out_dtype`` rounds the float32 result inside the kernel: the same bits as the float32 norm
    followed by ``.to(dtype)``, forward and both gradients (the incoming gradient in ``dtype``), on
    the vector path (widths 512, 1024) and the scalar one (36)."""
    g = torch.Generator(device=CUDA).manual_seed(5)
    x = 3 * torch.randn(777, width, device=CUDA, generator=g)
    gain = 1 + 0.1 * torch.randn(width, device=CUDA, generator=g)
    up = torch.randn(777, width, device=CUDA, generator=g).to(dtype)
    outs = []
    for fused in (True, False):
        xs, w = x.clone().requires_grad_(), gain.clone().requires_grad_()
        y = fused_rms_norm(xs, w, FLOOR, EPS, dtype) if fused else fused_rms_norm(xs, w, FLOOR, EPS).to(dtype)
        assert y.dtype == dtype
        y.backward(up)
        outs.append((y.detach(), xs.grad, w.grad))
    for got, want in zip(*outs, strict=True):
        assert torch.equal(got, want)


@pytest.mark.parametrize(("rdtype", "out"), [(torch.bfloat16, torch.bfloat16), (torch.float32, None), (torch.float16, torch.float16)])
def test_residual_add_fused_with_the_norm_equals_the_add_then_the_norm(rdtype: torch.dtype, out) -> None:
    """``add_rms_norm`` (one kernel each way) gives the same bits as ``x + r`` followed by the
    norm: the sum, the norm, and the gradients of x, r and the gain when both the sum and the norm
    are read downstream (the column's residual stream)."""
    from vesper_b200.kernels.norm import add_rms_norm

    g = torch.Generator(device=CUDA).manual_seed(6)
    x = 3 * torch.randn(1000, 512, device=CUDA, generator=g)
    r = torch.randn(1000, 512, device=CUDA, generator=g).to(rdtype)
    gain = 1 + 0.1 * torch.randn(512, device=CUDA, generator=g)
    up_s = torch.randn(1000, 512, device=CUDA, generator=g)
    up_y = torch.randn(1000, 512, device=CUDA, generator=g).to(out or torch.float32)
    outs = []
    for fused in (True, False):
        xs, rs, w = x.clone().requires_grad_(), r.clone().requires_grad_(), gain.clone().requires_grad_()
        if fused:
            s, y = add_rms_norm(xs, rs, w, FLOOR, EPS, out)
        else:
            s = xs + rs
            y = fused_rms_norm(s, w, FLOOR, EPS, out)
        torch.autograd.backward([s, y], [up_s, up_y])
        outs.append((s.detach(), y.detach(), xs.grad, rs.grad, w.grad))
    for got, want in zip(*outs, strict=True):
        assert got.dtype == want.dtype
        assert torch.equal(got, want)
