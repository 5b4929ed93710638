"""The write strength fused into the scan (``from_logits``) on a B200, against ``write_strength``.

The reference forms ``beta = write_strength(logits)`` = ``sigmoid(logits)`` (or, with a
modulator, ``sigmoid(logits + ln(1 + alpha m))`` and an exact zero where ``1 + alpha m`` is zero;
vesper/recurrence.py:34-88) before the scan. Here the scan kernels form it from the logits. The
fused path must equal ``torch.sigmoid`` followed by the unfused scan BIT FOR BIT, forward and
backward, in bf16 and in fp32 (the same float32 sigmoid, the same rounding, the same
``sigmoid_backward`` order); the modulated form must match the reference's formula; and the whole
chain must match the float64 oracle fed ``beta = sigmoid(logits)``.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import max_rel, rel
from vesper_b200.kernels.delta_scan import (
    check_status,
    delta_scan_fused,
    delta_scan_fused_fp32,
    modulation_shift,
)

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")


def _inputs(b, n, h, d, dtype, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, n, h, d, generator=g)
    k = torch.nn.functional.normalize(torch.randn(b, n, h, d, generator=g), dim=-1)
    v = torch.randn(b, n, h, d, generator=g)
    logits = 2.0 * torch.randn(b, n, h, generator=g)
    s0 = 0.3 * torch.randn(b, h, d, d, generator=g)
    d_o = torch.randn(b, n, h, d, generator=g)
    d_s = torch.randn(b, h, d, d, generator=g)
    q, k, v, logits = (t.to(dtype).to(CUDA) for t in (q, k, v, logits))
    return q, k, v, logits, s0.to(CUDA), d_o.to(CUDA), d_s.to(CUDA)


def _run(kernel, q, k, v, beta_in, s0, d_o, d_s, *, fused: bool, shift=None, beta_fn=None):
    leaves = [t.detach().requires_grad_() for t in (q, k, v, beta_in, s0)]
    lq, lk, lv, lb, ls = leaves
    if fused:
        o, sn = kernel(lq, lk, lv, lb, ls, from_logits=True, shift=shift)
    else:
        o, sn = kernel(lq, lk, lv, beta_fn(lb), ls)
    ((o.float() * d_o).sum() + (sn * d_s).sum()).backward()
    check_status(CUDA)
    return [o.detach(), sn.detach()] + [t.grad for t in leaves]


@pytest.mark.parametrize(("kernel", "dtype"), [(delta_scan_fused, torch.bfloat16),
                                               (delta_scan_fused_fp32, torch.float32)],
                         ids=["bf16", "fp32"])  # fmt: skip
def test_fused_logits_equal_sigmoid_then_scan_bit_for_bit(kernel, dtype) -> None:
    q, k, v, logits, s0, d_o, d_s = _inputs(2, 200, 3, 64, dtype)
    fused = _run(kernel, q, k, v, logits, s0, d_o, d_s, fused=True)
    plain = _run(kernel, q, k, v, logits, s0, d_o, d_s, fused=False, beta_fn=torch.sigmoid)
    names = ("o", "state", "dq", "dk", "dv", "dlogits", "dstate0")
    for name, a, b in zip(names, fused, plain, strict=True):
        assert torch.equal(a, b), (name, (a.float() - b.float()).abs().max().item())


def test_modulated_write_strength_matches_the_reference_formula() -> None:
    # write_strength(logits, m, alpha) = where(1 + alpha m > 0, sigmoid(logits + ln(1 + alpha m)), 0)
    q, k, v, logits, s0, d_o, d_s = _inputs(2, 130, 2, 32, torch.float32, seed=3)
    g = torch.Generator().manual_seed(4)
    alpha = 0.5
    m = torch.rand(2, 130, generator=g) * 4 - 1.5
    m[0, 7] = -1.0 / alpha  # a zero factor: an exact zero write
    m[1, 64] = -1.0 / alpha
    m = m.to(CUDA)
    shift = modulation_shift(logits, m, alpha)

    def reference(lg: torch.Tensor) -> torch.Tensor:
        factor = 1.0 + alpha * m
        beta = torch.sigmoid(lg + torch.log(factor.clamp_min(torch.finfo(factor.dtype).tiny))[..., None])
        return torch.where((factor > 0)[..., None], beta, torch.zeros_like(beta))

    fused = _run(delta_scan_fused_fp32, q, k, v, logits, s0, d_o, d_s, fused=True, shift=shift)
    plain = _run(delta_scan_fused_fp32, q, k, v, logits, s0, d_o, d_s, fused=False, beta_fn=reference)
    names = ("o", "state", "dq", "dk", "dv", "dlogits", "dstate0")
    for name, a, b in zip(names, fused, plain, strict=True):
        assert rel(a.cpu().numpy(), b.cpu().numpy()) < 1e-6, (name, rel(a.cpu().numpy(), b.cpu().numpy()))
    dlogits = fused[5]
    assert torch.all(dlogits[0, 7] == 0) and torch.all(dlogits[1, 64] == 0)
    with pytest.raises(ValueError, match="must not be negative"):
        modulation_shift(logits, torch.full_like(m, -3.0), alpha)


def test_fused_logits_match_the_oracle_in_bf16() -> None:
    # the oracle fed beta = sigmoid(logits) in float64; the logits' gradient is dbeta beta (1 - beta)
    q, k, v, logits, s0, d_o, d_s = _inputs(2, 300, 4, 128, torch.bfloat16, seed=9)
    o, sn, dq, dk, dv, dl, ds0 = _run(delta_scan_fused, q, k, v, logits, s0, d_o, d_s, fused=True)
    lg = logits.double().cpu().numpy()
    beta = 1.0 / (1.0 + np.exp(-lg))
    args = [t.double().cpu().numpy() for t in (q, k, v)]
    o_w, s_w = oracle.delta_scan(*args, beta, s0.cpu().numpy())
    dq_w, dk_w, dv_w, db_w, ds_w = oracle.delta_scan_grads(*args, beta, s0.cpu().numpy(), d_o.cpu().numpy(),
                                                           d_s.cpu().numpy())  # fmt: skip
    for name, got, want in (("o", o, o_w), ("state", sn, s_w), ("dq", dq, dq_w), ("dk", dk, dk_w), ("dv", dv, dv_w),
                            ("dlogits", dl, db_w * beta * (1.0 - beta)), ("dstate0", ds0, ds_w)):  # fmt: skip
        a = got.float().cpu().numpy()
        assert rel(a, want) < 1.5e-2 and max_rel(a, want) < 2e-2, (name, rel(a, want), max_rel(a, want))
