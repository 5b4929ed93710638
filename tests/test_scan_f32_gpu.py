"""``delta_scan_fused_fp32`` on a B200 against the reference (golden vectors) and the oracle.

The float32 kernel's licence is float32 rounding only: 1e-5 relative (the reference's TOL_FP32,
vesper tests/test_delta_scan_fused.py:255) on outputs, the final state and all five gradients, at
the reference's test sizes, at config 1 (2 x 512 x 4 x 64) and at 4096 tokens.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import golden, golden_names, rel
from vesper_b200.contracts import ContractError
from vesper_b200.kernels.delta_scan import delta_scan_fused_fp32

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")
TOL_FP32 = 1e-5


def _inputs(b, n, h, d, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, n, h, d, generator=g)
    k = torch.randn(b, n, h, d, generator=g)
    k = k / k.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    v = torch.randn(b, n, h, d, generator=g)
    beta = torch.sigmoid(torch.randn(b, n, h, generator=g))
    s0 = 0.5 * torch.randn(b, h, d, d, generator=g)
    return q, k, v, beta, s0


def _fwd_bwd(q, k, v, beta, s0, d_o, d_s):
    ins = [t.to(CUDA).requires_grad_() for t in (q, k, v, beta, s0)]
    o, s = delta_scan_fused_fp32(*ins)
    ((o * d_o.to(CUDA)).sum() + (s * d_s.to(CUDA)).sum()).backward()
    return o.detach().cpu().numpy(), s.detach().cpu().numpy(), [t.grad.cpu().numpy() for t in ins]


@pytest.mark.parametrize("name", golden_names("scan_"))
def test_forward_state_and_gradients_equal_the_reference(name: str) -> None:
    f = golden(name)
    q, k, v, beta, h0, d_o, d_s = (torch.from_numpy(f[x]) for x in ("q", "k", "v", "beta", "h0", "d_o", "d_s"))
    o, s, grads = _fwd_bwd(q, k, v, beta, h0, d_o, d_s)
    assert rel(o, f["o"]) < TOL_FP32
    assert rel(s, f["s"]) < TOL_FP32
    for got, key in zip(grads, ("dq", "dk", "dv", "dbeta", "dh0"), strict=True):
        assert rel(got, f[key]) < TOL_FP32, key


@pytest.mark.parametrize(("b", "n", "h", "d"), [(2, 512, 4, 64), (1, 4096, 2, 64), (2, 200, 2, 128), (1, 70, 1, 256)])
def test_config_sizes_equal_the_oracle(b: int, n: int, h: int, d: int) -> None:
    q, k, v, beta, s0 = _inputs(b, n, h, d)
    g = torch.Generator().manual_seed(7)
    d_o, d_s = torch.randn(b, n, h, d, generator=g), torch.randn(b, h, d, d, generator=g)
    o, s, grads = _fwd_bwd(q, k, v, beta, s0, d_o, d_s)
    o_w, s_w = oracle.delta_scan(*(t.numpy() for t in (q, k, v, beta, s0)))
    g_w = oracle.delta_scan_grads(*(t.numpy() for t in (q, k, v, beta, s0, d_o, d_s)))
    assert rel(o, o_w) < TOL_FP32
    assert rel(s, s_w) < TOL_FP32
    for got, want, key in zip(grads, g_w, ("dq", "dk", "dv", "dbeta", "ds0"), strict=True):
        assert rel(got, want) < TOL_FP32, key


def test_a_carried_state_continues_the_sequence_and_no_tokens_change_nothing() -> None:
    q, k, v, beta, s0 = (t.to(CUDA) for t in _inputs(2, 130, 3, 16))
    o_ref, s_ref = delta_scan_fused_fp32(q, k, v, beta, s0)
    o_a, s_a = delta_scan_fused_fp32(q[:, :50], k[:, :50], v[:, :50], beta[:, :50], s0)
    o_b, s_b = delta_scan_fused_fp32(q[:, 50:], k[:, 50:], v[:, 50:], beta[:, 50:], s_a)
    assert rel(torch.cat([o_a, o_b], 1).cpu().numpy(), o_ref.cpu().numpy()) < TOL_FP32
    assert rel(s_b.cpu().numpy(), s_ref.cpu().numpy()) < TOL_FP32
    o0, s0_out = delta_scan_fused_fp32(q[:, :0], k[:, :0], v[:, :0], beta[:, :0], s0)
    assert o0.shape == (2, 0, 3, 16)
    assert s0_out is s0


def test_gradients_flow_from_a_state_that_needs_none() -> None:
    q, k, v, beta, s0 = _inputs(2, 63, 3, 16)
    ins = [t.to(CUDA).requires_grad_() for t in (q, k, v, beta)]
    state = s0.to(CUDA)
    o, _ = delta_scan_fused_fp32(*ins, state)
    o.square().sum().backward()
    assert state.grad is None and not state.requires_grad
    o_w, _ = oracle.delta_scan(*(t.numpy() for t in (q, k, v, beta, s0)))
    g_w = oracle.delta_scan_grads(*(t.numpy() for t in (q, k, v, beta, s0)), 2 * o_w, np.zeros(s0.shape))
    for t, want in zip(ins, g_w[:4], strict=True):
        assert rel(t.grad.cpu().numpy(), want) < TOL_FP32


def test_refuses_bfloat16_inputs_and_a_cpu_state() -> None:
    q, k, v, beta, s0 = (t.to(CUDA) for t in _inputs(1, 8, 2, 16))
    with pytest.raises(ContractError, match="dtype"):
        delta_scan_fused_fp32(q.bfloat16(), k, v, beta, s0)
    with pytest.raises(ContractError, match="is on cpu"):
        delta_scan_fused_fp32(q, k, v, beta, s0.cpu())
    with pytest.raises(ContractError, match="exceeds"):
        w = torch.zeros(1, 4, 1, 512, device=CUDA)
        delta_scan_fused_fp32(w, w, w, torch.zeros(1, 4, 1, device=CUDA), torch.zeros(1, 1, 512, 512, device=CUDA))
