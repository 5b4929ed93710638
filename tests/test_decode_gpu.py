"""Batched one-token decoding (``vesper_b200.decode``) on a B200 against the reference's decoder.

The fixture ``decode_greedy`` is the reference's own ``decode_step`` semantics (the loop at depth 2
under ``DenseRule`` over ``RingKVCache`` windows, the head on each token; vesper/decode.py:29-46)
fed two rows token by token in float64: each row's 24-token prompt, then 8 greedy tokens. Here the
two rows decode together: the prompt through the chunked prefill, then one captured step per
token. In float32 every logit agrees to float32 rounding and every greedy id is the reference's;
in bf16 to bf16 rounding. The two kernels of the step are checked alone: the one-token scan against
the float64 oracle, the ring attention against a masked softmax written out in torch.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import golden, rel
from vesper_b200 import _lib
from vesper_b200.attention import WindowedAttention, kv_ring_empty
from vesper_b200.column import ColumnShape, set_scan
from vesper_b200.decode import BatchedDecoder
from vesper_b200.kernels.delta_scan import delta_scan_step_
from vesper_b200.model import Vesper

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")
SHAPE = ColumnShape(d=64, heads=2, kv_groups=2, head_dim=32, window=16, rotary_base=10000.0, ffn_mult=2,
                    block=16, key_conv=4)  # fmt: skip


def _model(f: dict[str, np.ndarray]) -> Vesper:
    model = Vesper(SHAPE, int(f["vocab"]), int(f["columns"]), int(f["t_max"]), 0.01, torch.Generator().manual_seed(7))
    assert abs(float(model.embedding.weight.double().sum()) - float(f["sum.embedding.weight"])) < 1e-9
    for k, p in model.loop.named_parameters():
        if k != "u":
            assert abs(float(p.detach().double().sum()) - float(f[f"sum.{k}"])) <= 1e-9 * max(1.0, abs(float(f[f"sum.{k}"]))), k
    with torch.no_grad():
        model.loop.u.copy_(torch.from_numpy(f["u"]).float())
    return model.to(CUDA)


def _decode(f, dtype, scan: str):
    model = _model(f)
    set_scan(model, scan)
    prompt, gen, depth, vocab = int(f["prompt"]), int(f["gen"]), int(f["depth"]), int(f["vocab"])
    tokens = torch.from_numpy(f["tokens"]).to(CUDA)
    dec = BatchedDecoder(model, depth, vocab, b=tokens.shape[0], dtype=dtype, warm=2)
    pre = dec.prefill(tokens[:, :prompt], chunk=10, all_logits=True)
    logits, ids = [pre.float()], []
    for i in range(gen):
        nid, lg = dec.step(tokens[:, prompt + i : prompt + i + 1])
        logits.append(lg.float().clone())
        ids.append(nid.clone())
    _lib.check_status(CUDA)
    dec.release()
    return torch.cat(logits, 1).double().cpu().numpy(), torch.cat(ids, 1).cpu().numpy()


def test_float32_decoding_matches_the_reference_decoder_token_for_token() -> None:
    f = golden("decode_greedy")
    logits, ids = _decode(f, torch.float32, "fused-fp32")
    want = f["logits"]
    assert logits.shape == want.shape
    for row in range(want.shape[0]):
        assert rel(logits[row], want[row]) < 1e-5, (row, rel(logits[row], want[row]))
    prompt = int(f["prompt"])
    assert np.array_equal(ids[:, :-1], f["tokens"][:, prompt + 1 :])


def test_bf16_decoding_matches_the_reference_decoder_to_bf16_rounding() -> None:
    f = golden("decode_greedy")
    logits, _ = _decode(f, torch.bfloat16, "fused")
    want = f["logits"]
    for row in range(want.shape[0]):
        assert rel(logits[row], want[row]) < 3e-2, (row, rel(logits[row], want[row]))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_the_one_token_scan_matches_the_oracle(dtype: torch.dtype) -> None:
    b, h, d = 5, 3, 64
    g = torch.Generator().manual_seed(3)
    q = torch.randn(b, 1, h, d, generator=g).to(dtype)
    k = torch.nn.functional.normalize(torch.randn(b, 1, h, d, generator=g), dim=-1).to(dtype)
    v = torch.randn(b, 1, h, d, generator=g).to(dtype)
    logits = torch.randn(b, 1, h, generator=g).to(dtype)
    s0 = 0.5 * torch.randn(b, h, d, d, generator=g)
    state = s0.to(CUDA).clone()
    o = delta_scan_step_(*(t.to(CUDA) for t in (q, k, v, logits)), state, from_logits=True)
    beta = torch.sigmoid(logits.float()).to(dtype).double().numpy()
    o_w, s_w = oracle.delta_scan(*(t.double().numpy() for t in (q, k, v)), beta, s0.double().numpy())
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    assert rel(o.float().cpu().numpy(), o_w) < tol and rel(state.cpu().numpy(), s_w) < tol


def test_the_ring_attention_matches_a_masked_softmax_and_writes_its_slot() -> None:
    b, heads, kv_groups, dk, window = 4, 8, 4, 64, 16
    attn = WindowedAttention(64, heads, kv_groups, dk, window, 10000.0, torch.Generator().manual_seed(1)).to(CUDA)
    hkv = heads // kv_groups
    g = torch.Generator(device=CUDA).manual_seed(2)
    ring = kv_ring_empty(b, hkv, dk, window, torch.float32, CUDA)
    ring.k.copy_(torch.randn(ring.k.shape, device=CUDA, generator=g))
    ring.v.copy_(torch.randn(ring.v.shape, device=CUDA, generator=g))
    pos = torch.tensor([[40], [41], [3], [100]], device=CUDA)
    # slot contents: positions p - 20 .. p - 1 scattered, some invalid, some out of the window
    for r in range(b):
        for s_ in range(window):
            ring.pos[r, s_] = max(0, int(pos[r]) - 1 - ((s_ * 7 + r) % 20))
        ring.valid[r] = torch.rand(window, device=CUDA, generator=g) < 0.8
    q = torch.randn(b, 1, heads, dk, device=CUDA, generator=g)
    k = torch.randn(b, 1, hkv, dk, device=CUDA, generator=g)
    v = torch.randn(b, 1, hkv, dk, device=CUDA, generator=g)
    before = (ring.k.clone(), ring.v.clone(), ring.pos.clone(), ring.valid.clone())
    # the masked softmax over ring + itself, written out
    keys = torch.cat([before[0], k], 1)
    vals = torch.cat([before[1], v], 1)
    kpos = torch.cat([before[2], pos], 1)
    valid = torch.cat([before[3], torch.ones_like(before[3][:, :1])], 1)
    allowed = valid & (kpos <= pos) & (kpos > pos - window)
    own = (pos % window)
    allowed[torch.arange(b), own[:, 0]] = False  # the slot being replaced is never visible
    rep = heads // hkv
    kx = keys.repeat_interleave(rep, dim=2)
    vx = vals.repeat_interleave(rep, dim=2)
    sc = torch.einsum("bhd,blhd->bhl", q[:, 0], kx) / dk**0.5
    sc = sc.masked_fill(~allowed[:, None, :], float("-inf"))
    want = torch.einsum("bhl,blhd->bhd", torch.softmax(sc, -1), vx)
    y, _ = attn.attend_ring(q, k, v, pos, ring)
    want_y = attn.output(want[:, None])
    assert rel(y.detach().cpu().numpy(), want_y.detach().cpu().numpy()) < 1e-5
    idx = torch.arange(b, device=CUDA)
    assert torch.equal(ring.k[idx, own[:, 0]], k[:, 0]) and torch.equal(ring.v[idx, own[:, 0]], v[:, 0])
    assert torch.equal(ring.pos[idx, own[:, 0]], pos[:, 0]) and bool(ring.valid[idx, own[:, 0]].all())
    _lib.check_status(CUDA)
