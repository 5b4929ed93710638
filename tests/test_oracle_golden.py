"""The CPU oracle against the reference's own results (golden vectors) and its known answers.

tests/golden/make_golden.py produced the fixtures by running the reference's pure-PyTorch path in
float64; the oracle (a C restatement) must reproduce every value and gradient to float64
rounding. The two-token rational known-answer test is the reference's own hand derivation
(tests/test_recurrence_review.py:9-37 of the reference), reused as numbers.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import golden, golden_names, rel

TOL = 1e-10


def test_two_token_rational_known_answer() -> None:
    q = np.array([[2.0, -1.0], [-1.0, 3.0]]).reshape(1, 2, 1, 2)
    k = np.array([[3 / 5, 4 / 5], [0.0, 1.0]]).reshape(1, 2, 1, 2)
    v = np.array([[5.0, -2.0], [-3.0, 1.0]]).reshape(1, 2, 1, 2)
    beta = np.array([1 / 2, 3 / 4]).reshape(1, 2, 1)
    h0 = np.array([[1.0, 2.0], [3.0, 4.0]]).reshape(1, 1, 2, 2)
    h2 = np.array([[8 / 5, 2 / 25], [-13 / 10, 111 / 100]]).reshape(1, 1, 2, 2)
    expected = np.array([[-3 / 5, -32 / 25], [-11 / 2, 13 / 4]]).reshape(1, 2, 1, 2)
    o, s = oracle.delta_scan(q, k, v, beta, h0)
    np.testing.assert_allclose(o, expected, rtol=0, atol=1e-12)
    np.testing.assert_allclose(s, h2, rtol=0, atol=1e-12)
    h1 = np.array([[8 / 5, 2 / 25], [19 / 5, 36 / 25]]).reshape(1, 1, 2, 2)
    _, s1 = oracle.delta_scan(q[:, :1], k[:, :1], v[:, :1], beta[:, :1], h0)
    np.testing.assert_allclose(s1, h1, rtol=0, atol=1e-12)


@pytest.mark.parametrize("name", golden_names("scan_"))
def test_scan_forward_and_gradients_equal_the_reference(name: str) -> None:
    f = golden(name)
    o, s = oracle.delta_scan(f["q"], f["k"], f["v"], f["beta"], f["h0"])
    assert rel(o, f["o"]) < TOL
    assert rel(s, f["s"]) < TOL
    grads = oracle.delta_scan_grads(f["q"], f["k"], f["v"], f["beta"], f["h0"], f["d_o"], f["d_s"])
    for got, key in zip(grads, ("dq", "dk", "dv", "dbeta", "dh0"), strict=True):
        assert rel(got, f[key]) < TOL, key


@pytest.mark.parametrize("name", golden_names("keys_"))
def test_key_filter_and_gradients_equal_the_reference(name: str) -> None:
    f = golden(name)
    heads = int(f["heads"])
    k = oracle.keys(f["z"], f["hist"], f["taps"], heads)
    assert rel(k, f["k"]) < TOL
    np.testing.assert_array_equal(oracle.next_history(f["z"], f["hist"]), f["next_hist"])
    dz, dhist, dtaps = oracle.keys_grads(f["z"], f["hist"], f["taps"], heads, f["up"])
    assert rel(dz, f["dz"]) < TOL
    assert rel(dhist, f["dhist"]) < TOL
    assert rel(dtaps, f["dtaps"]) < TOL


@pytest.mark.parametrize("name", golden_names("norm_"))
def test_rms_norm_and_gradients_equal_the_reference(name: str) -> None:
    f = golden(name)
    y, _ = oracle.rms_norm(f["x"], f["gain"])
    np.testing.assert_allclose(y, f["y"], rtol=1e-12, atol=1e-300)
    dx, dg = oracle.rms_norm_grads(f["x"], f["gain"], f["up"])
    np.testing.assert_allclose(dx, f["dx"], rtol=1e-9, atol=1e-300)
    np.testing.assert_allclose(dg, f["dg"], rtol=1e-9, atol=1e-12)


def test_rms_norm_boundary_values_hold() -> None:
    f = golden("norm_boundary")
    y, _ = oracle.rms_norm(f["x"], f["gain"])
    assert np.isfinite(y).all()
    assert y[2, 0] == pytest.approx(0.0995, abs=5e-5)  # eps regularizes, does not floor
    assert np.abs(y[1]).max() == 0.0


@pytest.mark.parametrize("name", golden_names("attn_"))
def test_window_attention_and_gradients_equal_the_reference(name: str) -> None:
    f = golden(name)
    w = int(f["window"])
    keys = np.concatenate([f["ck"], f["k"]], axis=1)
    vals = np.concatenate([f["cv"], f["v"]], axis=1)
    o = oracle.window_attention(f["q"], keys, vals, w)
    assert rel(o, f["o"]) < TOL
    dq, dk, dv = oracle.window_attention_grads(f["q"], keys, vals, w, f["up"])
    m = f["ck"].shape[1]
    assert rel(dq, f["dq"]) < TOL
    assert rel(dk[:, m:], f["dk"]) < TOL
    assert rel(dv[:, m:], f["dv"]) < TOL
    if m:
        assert rel(dk[:, :m], f["dck"]) < TOL
        assert rel(dv[:, :m], f["dcv"]) < TOL
