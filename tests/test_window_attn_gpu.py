"""``window_attention`` (tcgen05) on a B200 against the reference (golden) and the oracle.

The reference's own check (vesper tests/test_window_attn.py:62-75) compares its CUDA kernel with the
blocked CPU attention at rtol = atol = 3e-2 for the output and the gradients of q, k and v, with an
empty, a partly filled and a full cache; the golden fixtures are that blocked path run in float64
on bfloat16-valued inputs. At larger sizes the oracle (float64) is the truth, checked against the
north star's bfloat16 bound (2e-2 max-relative) and 1e-2 relative L2. The compacted form must give
the dense call's rows, and padding rows no output and no gradient.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import elem_rel, error_report, golden, golden_names, max_rel, rel
from vesper_b200 import _lib
from vesper_b200.contracts import ContractError
from vesper_b200.kernels.window_attn import window_attention, window_attention_active

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")
BF16 = torch.bfloat16


def _run(q, keys, values, window, d_o, qpos=None, counts=None):
    """Outputs and gradients through the public call, as float64 numpy arrays."""
    q, keys, values = (t.to(CUDA).detach().requires_grad_() for t in (q, keys, values))
    if qpos is None:
        o = window_attention(q, keys, values, window)
    else:
        o = window_attention_active(q, qpos.to(CUDA), None if counts is None else counts.to(CUDA), keys, values, window)
    assert o.dtype == q.dtype and o.shape == q.shape
    (o.float() * d_o.to(CUDA)).sum().backward()
    _lib.check_status(CUDA)
    out = [o.detach(), q.grad, keys.grad, values.grad]
    return [t.double().cpu().numpy() for t in out]


@pytest.mark.parametrize("name", golden_names("attn_"))
def test_output_and_gradients_match_the_reference(name: str) -> None:
    f = golden(name)
    window = int(f["window"])
    q = torch.from_numpy(f["q"]).to(BF16)
    keys = torch.from_numpy(np.concatenate([f["ck"], f["k"]], axis=1)).to(BF16)
    values = torch.from_numpy(np.concatenate([f["cv"], f["v"]], axis=1)).to(BF16)
    m = f["ck"].shape[1]
    o, dq, dkeys, dvalues = _run(q, keys, values, window, torch.from_numpy(f["up"]))
    pairs = [
        (o, f["o"], "o"), (dq, f["dq"], "dq"), (dkeys[:, m:], f["dk"], "dk"),
        (dvalues[:, m:], f["dv"], "dv"), (dkeys[:, :m], f["dck"], "dcache_k"),
        (dvalues[:, :m], f["dcv"], "dcache_v"),
    ]  # fmt: skip
    for got, want, what in pairs:
        torch.testing.assert_close(torch.from_numpy(got), torch.from_numpy(want), rtol=3e-2, atol=3e-2, msg=what)
        if want.size:
            assert rel(got, want) < 1e-2, (what, rel(got, want))


def _inputs(b, n, m, h, hkv, dk, seed, dtype=BF16):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(b, n, h, dk, generator=g).to(dtype)
    keys = torch.randn(b, m + n, hkv, dk, generator=g).to(dtype)
    values = torch.randn(b, m + n, hkv, dk, generator=g).to(dtype)
    d_o = torch.randn(b, n, h, dk, generator=g)
    return q, keys, values, d_o


def _oracle(q, keys, values, window, d_o):
    f64 = [t.double().numpy() for t in (q, keys, values, d_o)]
    o = oracle.window_attention(f64[0], f64[1], f64[2], window)
    return [o, *oracle.window_attention_grads(f64[0], f64[1], f64[2], window, f64[3])]


def _assert_matches(got, want, names=("o", "dq", "dkeys", "dvalues")):
    for a, b, what in zip(got, want, names, strict=True):
        print(f"{what}: {error_report(a, b)}")
        assert rel(a, b) < 1e-2, (what, rel(a, b))
        assert max_rel(a, b) < 2e-2, (what, max_rel(a, b))
        assert elem_rel(a, b) < 1e-1, (what, elem_rel(a, b))


@pytest.mark.parametrize(
    ("b", "n", "m", "window"),
    [(2, 700, 0, 512), (2, 600, 300, 512), (1, 1000, 512, 512), (2, 333, 17, 100), (2, 300, 5, 16), (3, 129, 0, 1)],
)
def test_config_3_geometry_matches_the_oracle(b: int, n: int, m: int, window: int) -> None:
    """8 query heads over 2 key heads of 64 channels (the column's attention), windows 1 to 512."""
    q, keys, values, d_o = _inputs(b, n, m, 8, 2, 64, seed=n + m + window)
    _assert_matches(_run(q, keys, values, window, d_o), _oracle(q, keys, values, window, d_o))


@pytest.mark.parametrize("dk", [16, 32, 48, 80, 96, 112, 128])
def test_every_head_dimension_matches_the_oracle(dk: int) -> None:
    q, keys, values, d_o = _inputs(2, 200, 40, 4, 2, dk, seed=dk)
    _assert_matches(_run(q, keys, values, 64, d_o), _oracle(q, keys, values, 64, d_o))


def test_float16_inputs_match_the_oracle() -> None:
    q, keys, values, d_o = _inputs(2, 300, 64, 4, 1, 64, seed=5, dtype=torch.float16)
    got = _run(q, keys, values, 128, d_o)
    _assert_matches(got, _oracle(q, keys, values, 128, d_o))


def test_the_compacted_rows_equal_the_dense_rows_and_padding_is_inert() -> None:
    b, n, m, h, hkv, dk, window = 3, 700, 64, 8, 2, 64, 256
    q, keys, values, d_o = _inputs(b, n, m, h, hkv, dk, seed=11)
    g = torch.Generator().manual_seed(12)
    active = torch.rand(b, n, generator=g) < torch.tensor([[0.6], [0.05], [0.0]])
    counts = active.sum(1).to(torch.int32)
    cap = 512
    qc = torch.zeros(b, cap, h, dk, dtype=BF16)
    dc = torch.zeros(b, cap, h, dk)
    qpos = torch.full((b, cap), -7, dtype=torch.int32)  # padding positions are never read
    d_dense = torch.zeros_like(d_o)
    for i in range(b):
        idx = active[i].nonzero().flatten()
        qc[i, : len(idx)] = q[i, idx]
        dc[i, : len(idx)] = d_o[i, idx]
        qpos[i, : len(idx)] = (idx + m).to(torch.int32)
        d_dense[i, idx] = d_o[i, idx]
    dense = _run(q, keys, values, window, d_dense)
    comp = _run(qc, keys, values, window, dc, qpos=qpos, counts=counts)
    for i in range(b):
        c = int(counts[i])
        idx = active[i].nonzero().flatten().numpy()
        for got, want, what in ((comp[0], dense[0], "o"), (comp[1], dense[1], "dq")):
            if c:
                assert max_rel(got[i, :c], want[i, idx]) < 1e-2, (what, i)
            assert not np.any(got[i, c:]), (what, "padding", i)
    for got, want, what in ((comp[2], dense[2], "dkeys"), (comp[3], dense[3], "dvalues")):
        assert max_rel(got, want) < 2e-2, what
        assert not np.any(got[2]), (what, "a batch row with no live query")


def test_a_chunk_of_zero_queries_returns_an_empty_output() -> None:
    q = torch.zeros(2, 0, 4, 16, dtype=BF16, device=CUDA)
    keys = torch.zeros(2, 5, 2, 16, dtype=BF16, device=CUDA)
    assert window_attention(q, keys, keys, 8).shape == (2, 0, 4, 16)


def test_contract_violations_are_refused_before_any_launch() -> None:
    q = torch.zeros(1, 8, 4, 64, dtype=BF16, device=CUDA)
    kv = torch.zeros(1, 8, 2, 64, dtype=BF16, device=CUDA)
    with pytest.raises(ContractError, match="dtype"):
        window_attention(q.double(), kv.double(), kv.double(), 8)
    with pytest.raises(ContractError, match="dtype"):
        window_attention(q.float(), kv, kv, 8)
    with pytest.raises(ContractError, match="CUDA only"):
        window_attention(q.cpu(), kv.cpu(), kv.cpu(), 8)
    with pytest.raises(ContractError, match="multiple of 16"):
        window_attention(q[..., :24].contiguous(), kv[..., :24].contiguous(), kv[..., :24].contiguous(), 8)
    with pytest.raises(ContractError, match="key heads"):
        window_attention(q[:, :, :3].contiguous(), kv, kv, 8)
    with pytest.raises(ContractError, match="window"):
        window_attention(q, kv, kv, 0)
    with pytest.raises(ContractError, match="fewer"):
        window_attention(q, kv[:, :4], kv[:, :4], 8)


def test_repeats_bitwise_and_equals_itself_captured() -> None:
    q, keys, values, d_o = _inputs(2, 500, 100, 8, 2, 64, seed=3)
    q, keys, values, d_o = (t.to(CUDA) for t in (q, keys, values, d_o))
    qs, ks, vs = (t.clone().requires_grad_() for t in (q, keys, values))

    def step():
        for t in (qs, ks, vs):
            t.grad = None
        o = window_attention(qs, ks, vs, 512)
        (o.float() * d_o).sum().backward()
        return [o.detach().clone(), qs.grad.clone(), ks.grad.clone(), vs.grad.clone()]

    eager = [step() for _ in range(2)]
    assert all(torch.equal(a, b) for a, b in zip(eager[0], eager[1], strict=True))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    for t in (qs, ks, vs):
        t.grad = None
    with torch.cuda.graph(graph):
        o = window_attention(qs, ks, vs, 512)
        (o.float() * d_o).sum().backward()
        out = [o, qs.grad, ks.grad, vs.grad]
    for _ in range(3):
        graph.replay()
        torch.cuda.synchronize()
        assert all(torch.equal(a, b) for a, b in zip(out, eager[0], strict=True))
    _lib.check_status(CUDA)


# ---- float32: the reference's float32 path, on CUDA cores at float32 rounding -----------------------

F32_TOL = 1e-5


@pytest.mark.parametrize("name", golden_names("attn_"))
def test_float32_output_and_gradients_match_the_reference_at_float32_rounding(name: str) -> None:
    f = golden(name)
    window = int(f["window"])
    q = torch.from_numpy(f["q"]).float()
    keys = torch.from_numpy(np.concatenate([f["ck"], f["k"]], axis=1)).float()
    values = torch.from_numpy(np.concatenate([f["cv"], f["v"]], axis=1)).float()
    m = f["ck"].shape[1]
    o, dq, dkeys, dvalues = _run(q, keys, values, window, torch.from_numpy(f["up"]))
    pairs = [(o, f["o"], "o"), (dq, f["dq"], "dq"), (dkeys[:, m:], f["dk"], "dk"), (dvalues[:, m:], f["dv"], "dv"),
             (dkeys[:, :m], f["dck"], "dcache_k"), (dvalues[:, :m], f["dcv"], "dcache_v")]  # fmt: skip
    for got, want, what in pairs:
        if want.size:
            assert rel(got, want) < F32_TOL, (what, rel(got, want))
            assert max_rel(got, want) < 1e-4, (what, max_rel(got, want))


@pytest.mark.parametrize(("b", "n", "m", "window", "dk"), [(2, 300, 0, 512, 64), (2, 200, 100, 64, 64),
                                                        (1, 130, 7, 1, 32), (2, 100, 20, 50, 128)])  # fmt: skip
def test_float32_matches_the_oracle(b: int, n: int, m: int, window: int, dk: int) -> None:
    q, keys, values, d_o = _inputs(b, n, m, 8, 2, dk, seed=n + window, dtype=torch.float32)
    got = _run(q, keys, values, window, d_o)
    for a, w, what in zip(got, _oracle(q, keys, values, window, d_o), ("o", "dq", "dkeys", "dvalues"), strict=True):
        assert rel(a, w) < F32_TOL, (what, rel(a, w))


def test_float32_compacted_rows_equal_the_dense_rows() -> None:
    b, n, m, h, hkv, dk, window = 2, 300, 32, 4, 2, 64, 100
    q, keys, values, d_o = _inputs(b, n, m, h, hkv, dk, seed=21, dtype=torch.float32)
    g = torch.Generator().manual_seed(22)
    active = torch.rand(b, n, generator=g) < torch.tensor([[0.5], [0.1]])
    counts = active.sum(1).to(torch.int32)
    qc = torch.zeros(b, n, h, dk)
    dc = torch.zeros(b, n, h, dk)
    qpos = torch.zeros(b, n, dtype=torch.int32)
    d_dense = torch.zeros_like(d_o)
    for i in range(b):
        idx = active[i].nonzero().flatten()
        qc[i, : len(idx)] = q[i, idx]
        dc[i, : len(idx)] = d_o[i, idx]
        qpos[i, : len(idx)] = (idx + m).to(torch.int32)
        d_dense[i, idx] = d_o[i, idx]
    dense = _run(q, keys, values, window, d_dense)
    comp = _run(qc, keys, values, window, dc, qpos=qpos, counts=counts)
    for i in range(b):
        c = int(counts[i])
        idx = active[i].nonzero().flatten().numpy()
        assert rel(comp[0][i, :c], dense[0][i, idx]) < F32_TOL and rel(comp[1][i, :c], dense[1][i, idx]) < F32_TOL
        assert not np.any(comp[0][i, c:]) and not np.any(comp[1][i, c:])
    assert rel(comp[2], dense[2]) < F32_TOL and rel(comp[3], dense[3]) < F32_TOL
