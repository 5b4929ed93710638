"""The fused squared ReLU and rotary kernels on a B200 against the reference's op sequences.

Both kernels claim the reference's arithmetic exactly: ``relu(z)`` then ``h * h`` in ``z``'s dtype
(vesper/ffn.py:44-56) and the rotary pair rotation with float64 phases cast to the activation dtype
(vesper/attention.py:178-217), forward and backward. The reference's torch op sequences run here
on the same device, and outputs and gradients must be equal bit for bit, in bfloat16 and float32.
"""

from __future__ import annotations

import pytest
import torch

from vesper_b200.kernels.act import relu_square
from vesper_b200.kernels.rotary import rotary

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")


def _rotary_reference(x, pos, base):
    """vesper/attention.py:178-217, the torch op sequence."""
    dk = x.shape[-1]
    half = dk // 2
    exponent = torch.arange(0, half, dtype=torch.float64, device=x.device) * (2.0 / dk)
    inv_freq = base ** (-exponent)
    angle = pos.to(torch.float64)[:, :, None] * inv_freq
    cos = angle.cos().to(x.dtype)[:, :, None, :]
    sin = angle.sin().to(x.dtype)[:, :, None, :]
    x1, x2 = x[..., 0::2], x[..., 1::2]
    return torch.stack([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).flatten(-2)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_relu_square_equals_relu_then_product(dtype: torch.dtype) -> None:
    g = torch.Generator().manual_seed(0)
    z = (3 * torch.randn(3, 77, 129, generator=g)).to(dtype).to(CUDA)
    z[0, 0, :5] = torch.tensor([0.0, -0.0, 1e-30, -1e-30, float("nan")], dtype=dtype)
    up = torch.randn(z.shape, generator=g).to(dtype).to(CUDA)
    a = z.clone().requires_grad_()
    ya = relu_square(a)
    ya.backward(up)
    b = z.clone().requires_grad_()
    h = torch.relu(b)
    yb = h * h
    yb.backward(up)
    assert torch.equal(ya, yb) or torch.equal(torch.nan_to_num(ya), torch.nan_to_num(yb))
    assert torch.equal(torch.nan_to_num(a.grad), torch.nan_to_num(b.grad))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize(("heads", "dk"), [(8, 64), (2, 32), (3, 128)])
def test_rotary_equals_the_reference_sequence(dtype: torch.dtype, heads: int, dk: int) -> None:
    g = torch.Generator().manual_seed(heads * dk)
    x = torch.randn(2, 301, heads, dk, generator=g).to(dtype).to(CUDA)
    pos = (torch.arange(301) + 70000).expand(2, 301).contiguous().to(CUDA)
    up = torch.randn(x.shape, generator=g).to(dtype).to(CUDA)
    a = x.clone().requires_grad_()
    ya = rotary(a, pos, 10000.0)
    ya.backward(up)
    b = x.clone().requires_grad_()
    yb = _rotary_reference(b, pos, 10000.0)
    yb.backward(up)
    assert torch.equal(ya, yb)
    assert torch.equal(a.grad, b.grad)


@pytest.mark.parametrize("fdtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("masked", [False, True])
def test_residual_add_with_halted_rows_zeroed_equals_the_add_then_the_zeroing(fdtype: torch.dtype, masked: bool) -> None:
    """``residual_add`` (one kernel each way) gives the same bits as ``x + f`` followed by the
    loop's zeroing of halted rows (``select_rows`` with nothing carried), values and gradients."""
    from vesper_b200.kernels.act import residual_add
    from vesper_b200.kernels.compact import select_rows

    g = torch.Generator().manual_seed(8)
    x = (3 * torch.randn(4, 300, 512, generator=g)).to(CUDA)
    f = torch.randn(4, 300, 512, generator=g).to(fdtype).to(CUDA)
    keep = (torch.rand(4, 300, generator=g) > 0.3).to(CUDA) if masked else None
    up = torch.randn(4, 300, 512, generator=g).to(CUDA)
    outs = []
    for fused in (True, False):
        xs, fs = x.clone().requires_grad_(), f.clone().requires_grad_()
        if fused:
            y = residual_add(xs, fs, keep)
        else:
            y = xs + fs
            if keep is not None:
                (y,) = select_rows(keep, [y], [None])
        y.backward(up)
        outs.append((y.detach(), xs.grad, fs.grad))
    for got, want in zip(*outs, strict=True):
        assert got.dtype == want.dtype
        assert torch.equal(got, want)
