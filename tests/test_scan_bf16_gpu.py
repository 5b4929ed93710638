"""``delta_scan_fused`` (bf16, tcgen05) on a B200 against the reference (golden) and the oracle.

The truth is the reference in float64 fed the same bfloat16-valued inputs. The kernel's licence is
its bfloat16 intermediates: the reference's bound is 1.5e-2 relative L2 on outputs, the final state
and all five gradients (vesper tests/test_delta_scan_fused.py:34), and the north star's is 2e-2
max-relative (largest error over the largest reference magnitude); both are checked, and the
per-element reading (each error against max(|want|, rms(want))) within 1e-1.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import elem_rel, error_report, golden, golden_names, max_rel, rel
from vesper_b200.contracts import ContractError
from vesper_b200.kernels.delta_scan import check_status, delta_scan_fused

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")
BF16 = torch.bfloat16
TOL = 1.5e-2
TOL_MAX = 2e-2
ELEM_TOL = 1e-1  # per element against max(|want|, rms(want)): the far tail of the bf16 rounding


def _inputs(b, n, h, d, seed=0, state_scale=0.5):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, n, h, d, generator=g)
    k = torch.randn(b, n, h, d, generator=g)
    k = k / k.norm(dim=-1, keepdim=True).clamp_min(1e-6)
    v = torch.randn(b, n, h, d, generator=g)
    beta = torch.sigmoid(torch.randn(b, n, h, generator=g))
    s0 = state_scale * torch.randn(b, h, d, d, generator=g)
    q, k, v, beta = (t.to(BF16) for t in (q, k, v, beta))
    return q, k, v, beta, s0


def _fwd_bwd(q, k, v, beta, s0, d_o, d_s):
    ins = [t.to(CUDA).requires_grad_() for t in (q, k, v, beta, s0)]
    o, s = delta_scan_fused(*ins)
    assert o.dtype == BF16 and s.dtype == torch.float32
    ((o.float() * d_o.to(CUDA)).sum() + (s * d_s.to(CUDA)).sum()).backward()
    check_status(CUDA)
    return o.detach().float().cpu().numpy(), s.detach().cpu().numpy(), [t.grad.float().cpu().numpy() for t in ins]


def _assert_close(got, want, name):
    print(f"{name}: {error_report(got, want)}")
    assert rel(got, want) < TOL, (name, rel(got, want))
    assert max_rel(got, want) < TOL_MAX, (name, max_rel(got, want))
    assert elem_rel(got, want) < ELEM_TOL, (name, elem_rel(got, want))


@pytest.mark.parametrize("name", golden_names("scan_"))
def test_forward_state_and_every_gradient_match_the_reference(name: str) -> None:
    f = golden(name)
    q, k, v, beta = (torch.from_numpy(f[x]).to(BF16) for x in ("q", "k", "v", "beta"))
    h0, d_o, d_s = (torch.from_numpy(f[x]) for x in ("h0", "d_o", "d_s"))
    o, s, grads = _fwd_bwd(q, k, v, beta, h0, d_o, d_s)
    _assert_close(o, f["o"], "o")
    _assert_close(s, f["s"], "state")
    for got, key in zip(grads, ("dq", "dk", "dv", "dbeta", "dh0"), strict=True):
        _assert_close(got, f[key], key)


@pytest.mark.parametrize(
    ("b", "n", "h", "d"), [(2, 512, 4, 64), (1, 4096, 2, 64), (2, 200, 2, 128), (2, 100, 3, 32), (1, 64, 1, 16)]
)
def test_config_sizes_match_the_oracle(b: int, n: int, h: int, d: int) -> None:
    q, k, v, beta, s0 = _inputs(b, n, h, d)
    g = torch.Generator().manual_seed(7)
    d_o, d_s = torch.randn(b, n, h, d, generator=g), torch.randn(b, h, d, d, generator=g)
    o, s, grads = _fwd_bwd(q, k, v, beta, s0, d_o, d_s)
    args = [t.float().numpy() for t in (q, k, v, beta, s0)]
    o_w, s_w = oracle.delta_scan(*args)
    g_w = oracle.delta_scan_grads(*args, d_o.numpy(), d_s.numpy())
    _assert_close(o, o_w, "o")
    _assert_close(s, s_w, "state")
    for got, want, key in zip(grads, g_w, ("dq", "dk", "dv", "dbeta", "ds0"), strict=True):
        _assert_close(got, want, key)


def test_config2_full_size_matches_the_oracle_on_sampled_sequences() -> None:
    # B=8, H=8, T=4096, d=128 (config 2): every sequence runs on the GPU; the oracle checks the
    # first and last batch rows (16 of the 64 sequences) at full length, outputs and gradients
    b, n, h, d = 8, 4096, 8, 128
    q, k, v, beta, s0 = _inputs(b, n, h, d, seed=11, state_scale=0.0)
    g = torch.Generator().manual_seed(12)
    d_o = torch.randn(b, n, h, d, generator=g)
    o, s, grads = _fwd_bwd(q, k, v, beta, s0, d_o, torch.zeros(b, h, d, d))
    for row in (0, b - 1):
        sl = slice(row, row + 1)
        args = [t[sl].float().numpy() for t in (q, k, v, beta, s0)]
        o_w, s_w = oracle.delta_scan(*args)
        g_w = oracle.delta_scan_grads(*args, d_o[sl].numpy(), np.zeros((1, h, d, d)))
        _assert_close(o[sl], o_w, "o")
        _assert_close(s[sl], s_w, "state")
        for got, want, key in zip(grads, g_w, ("dq", "dk", "dv", "dbeta", "ds0"), strict=True):
            _assert_close(got[sl], want, key)


@pytest.mark.parametrize("d", [256, 192, 20])
def test_head_dimensions_beyond_the_chunked_tiles_match_the_oracle(d: int) -> None:
    # the contract's dk <= 256 (vesper/kernels/delta_scan.py:28-31): widths the 128-wide chunked
    # tiles do not take run the token-serial float32 kernel, exact to float32 rounding
    b, n, h = 2, 150, 2
    q, k, v, beta, s0 = _inputs(b, n, h, d, seed=d)
    g = torch.Generator().manual_seed(d + 1)
    d_o, d_s = torch.randn(b, n, h, d, generator=g), torch.randn(b, h, d, d, generator=g)
    o, s, grads = _fwd_bwd(q, k, v, beta, s0, d_o, d_s)
    args = [t.float().numpy() for t in (q, k, v, beta, s0)]
    o_w, s_w = oracle.delta_scan(*args)
    g_w = oracle.delta_scan_grads(*args, d_o.numpy(), d_s.numpy())
    _assert_close(o, o_w, "o")
    _assert_close(s, s_w, "state")
    for got, want, key in zip(grads, g_w, ("dq", "dk", "dv", "dbeta", "ds0"), strict=True):
        _assert_close(got, want, key)


def test_a_carried_state_continues_the_sequence_and_no_tokens_change_nothing() -> None:
    q, k, v, beta, s0 = (t.to(CUDA) for t in _inputs(2, 130, 3, 16))
    o_ref, s_ref = delta_scan_fused(q, k, v, beta, s0)
    o_a, s_a = delta_scan_fused(q[:, :50], k[:, :50], v[:, :50], beta[:, :50], s0)
    o_b, s_b = delta_scan_fused(q[:, 50:], k[:, 50:], v[:, 50:], beta[:, 50:], s_a)
    args = [t.float().cpu().numpy() for t in (q, k, v, beta, s0)]
    o_w, s_w = oracle.delta_scan(*args)
    _assert_close(torch.cat([o_a, o_b], 1).float().cpu().numpy(), o_w, "o")
    _assert_close(s_b.cpu().numpy(), s_w, "state")
    o0, s0_out = delta_scan_fused(q[:, :0], k[:, :0], v[:, :0], beta[:, :0], s0)
    assert o0.shape == (2, 0, 3, 16)
    assert s0_out is s0


def test_refuses_what_the_kernel_was_not_built_for() -> None:
    q, k, v, beta, s0 = (t.to(CUDA) for t in _inputs(1, 8, 2, 16))
    with pytest.raises(ContractError, match="dtype"):
        delta_scan_fused(q.float(), k, v, beta, s0)
    with pytest.raises(ContractError, match="dtype"):
        delta_scan_fused(q, k, v, beta, s0.to(BF16))
    with pytest.raises(ContractError, match="axis"):
        delta_scan_fused(q, k[:, :4], v, beta, s0)
    with pytest.raises(ContractError, match="is on cpu"):
        delta_scan_fused(q, k, v, beta, s0.cpu())
    wide = torch.zeros(1, 8, 1, 512, dtype=BF16, device=CUDA)
    with pytest.raises(ContractError, match="exceeds"):
        delta_scan_fused(wide, wide, wide, torch.zeros(1, 8, 1, dtype=BF16, device=CUDA),
                         torch.zeros(1, 1, 512, 512, device=CUDA))


def test_captured_equals_eager_bitwise_and_repeats() -> None:
    q, k, v, beta, s0 = (t.to(CUDA) for t in _inputs(2, 300, 4, 64, seed=5))
    d_o = torch.randn(2, 300, 4, 64, device=CUDA)

    def step():
        ins = [t.detach().requires_grad_() for t in (q, k, v, beta, s0)]
        o, s = delta_scan_fused(*ins)
        ((o.float() * d_o).sum() + s.sum()).backward()
        return [o.detach().clone(), s.detach().clone()] + [t.grad.clone() for t in ins]

    eager = [step() for _ in range(2)]
    assert all(torch.equal(a, b) for a, b in zip(eager[0], eager[1], strict=True))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert all(torch.equal(a, b) for a, b in zip(out, eager[0], strict=True))
    check_status(CUDA)
