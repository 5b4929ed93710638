"""``Column.step`` with copy-forward and ``Loop.forward`` with halting on a B200 against the reference.

The fixtures are the reference's own column and loop (``vesper.column.Column``,
``vesper.loop.Loop``) in float64 on the CPU from its seeded initialization; the modules here draw
the same parameters from the same seed (checked by per-parameter sums). In float32 mode (the
``fused-fp32`` scan, float32 norms, key filter and attention) outputs, states and every gradient
agree within 1e-5 relative (L2), and the loop's pass counts are identical: every recorded halting
margin is far above float32 rounding. In bfloat16 mode (autocast, the chunked tcgen05 scan and
the attention kernel) a column is held to the north star's 2e-2 max-relative, the loop's output
(six column applications compounded) to 3e-2, and any pass count that differs must sit on a
decision within rounding of its threshold.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden, max_rel, rel
from vesper_b200 import _lib
from vesper_b200.attention import KVCache
from vesper_b200.column import Carry, Column, ColumnShape, ColumnState, Projections, init_column_state, set_scan
from vesper_b200.loop import CdfRule, HaltingHead, Loop

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")
SHAPE = ColumnShape(d=64, heads=2, kv_groups=2, head_dim=32, window=16, rotary_base=10000.0, ffn_mult=2,
                    block=16, key_conv=4)  # fmt: skip
SEED = 7
# The loop's output compounds six bfloat16 column applications (2 columns x 3 passes), each held to
# the north star's 2e-2 by the column test above: its bound is 3e-2 max-relative.
LOOP_BF16_MAX = 3e-2


def _t(a: np.ndarray, dtype: torch.dtype | None = torch.float32) -> torch.Tensor:
    t = torch.from_numpy(np.asarray(a)).to(CUDA)
    return t if dtype is None or not t.dtype.is_floating_point else t.to(dtype)


def _check_sums(module: torch.nn.Module, f: dict[str, np.ndarray]) -> None:
    for k, p in module.named_parameters():
        want = float(f[f"sum.{k}"])
        got = float(p.detach().double().sum())
        assert abs(got - want) <= 1e-9 * max(1.0, abs(want)), (k, got, want)


class _Report:
    """Every comparison of a test, asserted at the end so one run shows all the errors."""

    def __init__(self, tol: float, tol_max: float) -> None:
        self.tol, self.tol_max, self.rows, self.bad = tol, tol_max, [], []

    def __call__(self, got: torch.Tensor, want: np.ndarray, what: str) -> None:
        g = got.detach().double().cpu().numpy()
        assert g.shape == want.shape, (what, g.shape, want.shape)
        r, m = rel(g, want), max_rel(g, want)
        self.rows.append(f"{what}: rel {r:.2e} max_rel {m:.2e}")
        if not (r < self.tol and m < self.tol_max):
            self.bad.append(self.rows[-1])

    def check(self) -> None:
        print("\n".join(self.rows))
        assert not self.bad, self.bad


def _column_run(f: dict[str, np.ndarray], bf16: bool):
    col = Column(SHAPE, torch.Generator().manual_seed(SEED))
    _check_sums(col, f)
    col = col.to(CUDA)
    set_scan(col, "fused" if bf16 else "fused-fp32")
    names = ("x", "h1", "ck", "cv", "hist", "rec_z", "rec_k", "rec_v", "rec_beta", "attn_k", "attn_v")
    leaves = {k: _t(f[k]).requires_grad_() for k in names}
    b = leaves["x"].shape[0]
    cold = init_column_state(SHAPE, b, 2, torch.float32, CUDA)
    state = ColumnState(
        h=(cold.h[0], leaves["h1"]),
        kv=(cold.kv[0], KVCache(leaves["ck"], leaves["cv"], _t(f["cpos"], None), SHAPE.window)),
        key_history=(cold.key_history[0], leaves["hist"]),
    )
    active = _t(f["active"], None)
    proj = Projections(*(leaves[k] for k in ("rec_z", "rec_k", "rec_v", "rec_beta", "attn_k", "attn_v")))
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=bf16):
        y, new, written = col.step(leaves["x"], _t(f["pos"], None), state, 1, carry=Carry(active, proj))
    ((y.float() * _t(f["up"])).sum() + (new.h[1] * _t(f["up_h"])).sum()).backward()
    _lib.check_status(CUDA)
    return col, leaves, active, y, new, written


@pytest.mark.parametrize("bf16", [False, True], ids=["fp32", "bf16"])
def test_column_step_with_a_carry_matches_the_reference(bf16: bool) -> None:
    f = golden("column_step")
    _close = _Report(2e-2, 2e-2) if bf16 else _Report(1e-5, 1e-4)
    col, leaves, active, y, new, written = _column_run(f, bf16)
    act = f["active"]
    _close(y[active], f["y"][act], "y (active rows)")
    _close(new.h[1], f["h_new"], "state")
    _close(new.key_history[1], f["hist_next"], "key history")
    _close(new.kv[1].k, f["kv_k"], "cache k")
    _close(new.kv[1].v, f["kv_v"], "cache v")
    assert np.array_equal(new.kv[1].pos.cpu().numpy(), f["kv_pos"])
    for k, w in (("rec_z", "w_z"), ("rec_k", "w_k"), ("rec_v", "w_v"), ("rec_beta", "w_beta"),
                 ("attn_k", "w_ak"), ("attn_v", "w_av")):  # fmt: skip
        _close(getattr(written, k), f[w], f"written {k}")
    for k, t in leaves.items():
        _close(t.grad, f[f"dleaf.{k}"], f"grad {k}")
    for k, p in col.named_parameters():
        _close(p.grad, f[f"grad.{k}"], f"grad {k}")
    _close.check()


def _loop(f: dict[str, np.ndarray]) -> Loop:
    g = torch.Generator().manual_seed(SEED)
    cols = [Column(SHAPE, g) for _ in range(int(f["columns"]))]
    loop = Loop(cols, HaltingHead(SHAPE.d, g), SHAPE.d, int(f["t_max"]), 0.01)
    _check_sums(loop, f)
    with torch.no_grad():
        loop.halting.b_h.fill_(float(f["b_h"]))
        loop.halting.w_h.mul_(float(f["w_scale"]))
        loop.u.copy_(torch.from_numpy(f["u"]).float())
    return loop.to(CUDA)


def _loop_run(f: dict[str, np.ndarray], bf16: bool, loop: Loop | None = None):
    loop = _loop(f) if loop is None else loop
    set_scan(loop, "fused" if bf16 else "fused-fp32")
    x0 = _t(f["x0"]).requires_grad_()
    b, t_max = x0.shape[0], int(f["t_max"])
    states = [init_column_state(SHAPE, b, t_max, torch.float32, CUDA) for _ in range(int(f["columns"]))]
    rule = CdfRule(loop.halting, 0.5) if str(f["rule"]) == "cdf" else None
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=bf16):
        res = loop.forward(x0, _t(f["pos"], None), states, exit_rule=rule)
    ((res.y.float() * _t(f["up"])).sum() + 0.1 * res.ponder.float().sum()).backward()
    _lib.check_status(CUDA)
    return loop, x0, res


@pytest.mark.parametrize("name", ["loop_act", "loop_cdf"])
def test_loop_fp32_pass_counts_are_identical_and_values_match(name: str) -> None:
    f = golden(name)
    loop, x0, res = _loop_run(f, bf16=False)
    assert np.array_equal(res.n_iters.cpu().numpy(), f["n_iters"]), "pass counts"
    _close = _Report(1e-5, 1e-4)
    _close(res.y, f["y"], "y")
    _close(res.ponder, f["ponder"], "ponder")
    _close(res.per_pass, f["per_pass"].astype(np.float64), "per-pass outputs")
    _close(x0.grad, f["dx0"], "grad x0")
    for k, p in loop.named_parameters():
        if f"grad.{k}" in f:
            _close(p.grad, f[f"grad.{k}"].astype(np.float64), f"grad {k}")
    _close.check()


@pytest.mark.parametrize("name", ["loop_act", "loop_cdf"])
def test_loop_bf16_flips_only_at_the_threshold(name: str) -> None:
    f = golden(name)
    _, _, res = _loop_run(f, bf16=True)
    got, want = res.n_iters.cpu().numpy(), f["n_iters"]
    flips = got != want
    if flips.any():
        # the decision that differs is the one at pass min(got, want); its margin must be small
        t = np.minimum(got, want)[flips] - 1
        margins = np.abs(f["margins"][t, *np.nonzero(flips)])
        assert margins.max() < 3e-2, ("a pass count differs far from its threshold", margins.max())
    # a flipped token writes other projections into every later pass's states, and the scan and
    # the attention are causal: the positions before a row's first flip are unaffected by it
    y = res.y.detach().double().cpu().numpy()
    for row in range(got.shape[0]):
        first = int(np.argmax(flips[row])) if flips[row].any() else got.shape[1]
        if first:
            err = max_rel(y[row, :first], f["y"][row, :first])
            assert err < LOOP_BF16_MAX, (row, first, err)


def test_the_loop_step_repeats_bitwise_when_captured() -> None:
    f = golden("loop_act")
    loop = _loop(f)
    set_scan(loop, "fused")
    x0 = _t(f["x0"])
    pos = _t(f["pos"], None)
    up = _t(f["up"])
    b, t_max = x0.shape[0], int(f["t_max"])
    params = list(loop.parameters())

    def step():
        states = [init_column_state(SHAPE, b, t_max, torch.bfloat16, CUDA) for _ in range(int(f["columns"]))]
        with torch.autocast("cuda", dtype=torch.bfloat16):
            res = loop.forward(x0, pos, states)
        loss = (res.y.float() * up).sum() + 0.1 * res.ponder.float().sum()
        grads = torch.autograd.grad(loss, params)
        return [loss.detach(), res.n_iters, *grads]

    eager = [[t.clone() for t in step()] for _ in range(2)]
    assert all(torch.equal(a, c) for a, c in zip(eager[0], eager[1], strict=True))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        out = step()
    for _ in range(2):
        graph.replay()
        torch.cuda.synchronize()
        assert all(torch.equal(a, c) for a, c in zip(out, eager[0], strict=True))
    _lib.check_status(CUDA)
