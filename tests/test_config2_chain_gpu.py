"""The benchmarked config-2 step on a B200 against the oracle: RMSNorm -> key filter -> bf16 scan.

This is exactly the chain ``bench.py`` times (``fused_rms_norm`` -> ``fused_keys`` ->
``delta_scan_fused``, forward and backward) at BASELINE config 2's full size: B=8, H=8, T=4096,
d=128, width 1024. Unlike the bench it carries a nonzero initial state, a nonzero key history and
a nonzero state gradient, so every state path the column uses is exercised. As in the bench, the
scan takes the write-strength logits and forms beta = sigmoid(logits) in its kernels; the oracle
is fed the reference's write_strength of the same logits. The GPU runs all eight
batch rows; the float64 oracle (the reference's pure-PyTorch float32 path restated) checks two of
them in full: the output, the final state and the gradients of x, the gain, the taps, the history,
q, v, the logits and the initial state.

Bounds, the bf16 mode's: 1.5e-2 relative L2 (the reference's own test bound for its bf16 scan,
vesper tests/test_delta_scan_fused.py:34) and 2e-2 normwise max-relative (the north star's "max
relative", read as the largest error over the largest reference magnitude). Per element, against
``max(|want|, rms(want))``, a tensor of 33 M elements whose errors are bf16 rounding with a relative
L2 of about 5e-3 reaches 2e-2 to 8e-2 in its far tail (5 to 12 standard deviations); that reading
is asserted within ``ELEM_TOL`` = 1e-1 and every reading is printed.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import elem_rel, error_report, max_rel, rel
from vesper_b200.kernels.delta_scan import check_status, delta_scan_fused
from vesper_b200.kernels.keys import fused_keys
from vesper_b200.kernels.norm import fused_rms_norm

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")
BF16 = torch.bfloat16
B, T, H, D = 8, 4096, 8, 128
W = H * D
TAPS = 4
TOL, TOL_MAX = 1.5e-2, 2e-2
ELEM_TOL = 1e-1
ROWS = (0, B - 1)


def _inputs(seed: int = 21):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, W, generator=g).to(BF16)
    gain = 1.0 + 0.1 * torch.randn(W, generator=g)
    taps = 0.5 * torch.randn(TAPS, W, generator=g)
    hist = torch.randn(B, TAPS - 1, W, generator=g)
    q = torch.nn.functional.normalize(torch.randn(B, T, H, D, generator=g), dim=-1).to(BF16)
    v = torch.randn(B, T, H, D, generator=g).to(BF16)
    beta = torch.randn(B, T, H, generator=g).to(BF16)  # the write-strength logits
    s0 = 0.1 * torch.randn(B, H, D, D, generator=g)
    d_o = torch.randn(B, T, H, D, generator=g)
    d_s = torch.randn(B, H, D, D, generator=g)
    return x, gain, taps, hist, q, v, beta, s0, d_o, d_s


def test_config2_chain_forward_and_every_gradient_match_the_oracle() -> None:
    x, gain, taps, hist, q, v, beta, s0, d_o, d_s = _inputs()
    leaves = [t.to(CUDA).requires_grad_() for t in (x, gain, taps, hist, q, v, beta, s0)]
    lx, lg, lt, lh, lq, lv, lb, ls = leaves
    xn = fused_rms_norm(lx, lg, 1e-3, 1e-6)
    k = fused_keys(xn, lh, lt, H)
    o, sn = delta_scan_fused(lq, k, lv, lb, ls, from_logits=True)
    ((o.float() * d_o.to(CUDA)).sum() + (sn * d_s.to(CUDA)).sum()).backward()
    torch.cuda.synchronize()
    check_status(CUDA)
    got = {
        "o": o.detach().float().cpu().numpy(), "state": sn.detach().cpu().numpy(),
        "dx": lx.grad.float().cpu().numpy(), "dgain": lg.grad.cpu().numpy(),
        "dtaps": lt.grad.cpu().numpy(), "dhist": lh.grad.cpu().numpy(),
        "dq": lq.grad.float().cpu().numpy(), "dv": lv.grad.float().cpu().numpy(),
        "dlogits": lb.grad.float().cpu().numpy(), "ds0": ls.grad.cpu().numpy(),
    }  # fmt: skip
    del leaves, lx, lg, lt, lh, lq, lv, lb, ls, xn, k, o, sn
    rows = list(ROWS)
    # the oracle on the checked rows: the same bf16-valued inputs, float64 throughout
    xr = x[rows].double().numpy()
    g64, t64 = gain.double().numpy(), taps.double().numpy()
    hr = hist[rows].double().numpy()
    qr, vr, lr = (t[rows].double().numpy() for t in (q, v, beta))
    br = 1.0 / (1.0 + np.exp(-lr))  # write_strength
    sr, dor, dsr = s0[rows].double().numpy(), d_o[rows].double().numpy(), d_s[rows].double().numpy()
    xn_w, _ = oracle.rms_norm(xr, g64)
    k_w = oracle.keys(xn_w, hr, t64, H)
    o_w, s_w = oracle.delta_scan(qr, k_w, vr, br, sr)
    dq_w, dk_w, dv_w, db_w, ds_w = oracle.delta_scan_grads(qr, k_w, vr, br, sr, dor, dsr)
    dz_w, dh_w, dt_w = oracle.keys_grads(xn_w, hr, t64, H, dk_w)
    dx_w, dg_w = oracle.rms_norm_grads(xr, g64, dz_w)
    # every quantity here is a function of its own batch row; the gain's and the taps' gradients,
    # which sum over all rows, are checked by the next test on a batch of two rows
    want = {"o": o_w, "state": s_w, "dx": dx_w, "dhist": dh_w, "dq": dq_w, "dv": dv_w,
            "dlogits": db_w * br * (1.0 - br), "ds0": ds_w}  # fmt: skip
    report, bad = [], []
    for name, w in want.items():
        g_rows = got[name][rows]
        line = f"{name}: {error_report(g_rows, w)}"
        report.append(line)
        if not (rel(g_rows, w) < TOL and max_rel(g_rows, w) < TOL_MAX and elem_rel(g_rows, w) < ELEM_TOL):
            bad.append(line)
    print("\n".join(report))
    assert not bad, bad


def test_config2_chain_gain_and_taps_gradients_match_the_oracle_on_a_two_row_batch() -> None:
    # the parameter gradients sum over every row, so they are checked on a batch of the two rows
    x, gain, taps, hist, q, v, beta, s0, d_o, d_s = (t[list(ROWS)] if t.dim() > 2 and t.shape[0] == B else t
                                                     for t in _inputs(seed=22))  # fmt: skip
    leaves = [t.to(CUDA).requires_grad_() for t in (x, gain, taps, hist, q, v, beta, s0)]
    lx, lg, lt, lh, lq, lv, lb, ls = leaves
    xn = fused_rms_norm(lx, lg, 1e-3, 1e-6)
    k = fused_keys(xn, lh, lt, H)
    o, sn = delta_scan_fused(lq, k, lv, lb, ls, from_logits=True)
    ((o.float() * d_o.to(CUDA)).sum() + (sn * d_s.to(CUDA)).sum()).backward()
    torch.cuda.synchronize()
    check_status(CUDA)
    xr, g64, t64, hr = x.double().numpy(), gain.double().numpy(), taps.double().numpy(), hist.double().numpy()
    qr, vr, sr = (t.double().numpy() for t in (q, v, s0))
    br = 1.0 / (1.0 + np.exp(-beta.double().numpy()))
    xn_w, _ = oracle.rms_norm(xr, g64)
    k_w = oracle.keys(xn_w, hr, t64, H)
    _, dk_w, _, _, _ = oracle.delta_scan_grads(qr, k_w, vr, br, sr, d_o.double().numpy(), d_s.double().numpy())
    dz_w, _, dt_w = oracle.keys_grads(xn_w, hr, t64, H, dk_w)
    _, dg_w = oracle.rms_norm_grads(xr, g64, dz_w)
    report, bad = [], []
    for name, g_, w in (("dgain", lg.grad, dg_w), ("dtaps", lt.grad, dt_w)):
        a = g_.cpu().numpy()
        line = f"{name}: {error_report(a, w)}"
        report.append(line)
        if not (rel(a, w) < TOL and max_rel(a, w) < TOL_MAX and elem_rel(a, w) < ELEM_TOL):
            bad.append(line)
    print("\n".join(report))
    assert not bad, bad
