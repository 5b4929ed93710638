"""Generate the column and loop fixtures of tests/golden/ by running the reference itself.

Run in a container that holds the reference (mstampfli/vesper-preview) source:

    VESPER_REF=<reference checkout> PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden_loop.py

The reference's ``Column.step`` (with a copy-forward carry) and ``Loop.forward`` (ACT halting and
the CDF exit rule) run in float64 on the CPU, their pure-PyTorch path, from the reference's own
seeded initialization; gradients by autograd. Parameters are not stored: the build's modules
draw the same values from the same seed (each fixture keeps per-parameter sums to prove it).
Inputs are exactly representable in bfloat16 and stored as float32; results are float64. The
loop fixtures also keep every halting margin (``P + p - (1 - epsilon)``, or ``cdf - q``) so a
test can tell a real disagreement from a decision within rounding of its threshold.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
if "VESPER_REF" not in os.environ:
    sys.exit("set VESPER_REF to a checkout of the reference (mstampfli/vesper-preview)")
REF = Path(os.environ["VESPER_REF"])
sys.dont_write_bytecode = True
sys.path.insert(0, str(REF))

from vesper.attention import KVCache  # noqa: E402
from vesper.embedding import TiedEmbedding  # noqa: E402
from vesper.column import Carry, Column, ColumnShape, ColumnState, Projections  # noqa: E402
from vesper.loop import CdfRule, HaltingHead, Loop  # noqa: E402
from vesper.recurrence import normalize_keys  # noqa: E402

F64 = torch.float64
SHAPE = ColumnShape(d=64, heads=2, kv_groups=2, head_dim=32, window=16, rotary_base=10000.0, ffn_mult=2,
                    block=16, key_conv=4)  # fmt: skip
SEED = 7


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(F64)


def _save(name: str, **arrays: object) -> None:
    out: dict[str, np.ndarray] = {}
    for key, value in arrays.items():
        if isinstance(value, torch.Tensor):
            value = value.detach().cpu().numpy()
        out[key] = np.asarray(value)
    np.savez_compressed(HERE / f"{name}.npz", **out)


def _param_sums(module: torch.nn.Module) -> dict[str, np.ndarray]:
    return {f"sum.{k}": np.asarray(float(p.detach().double().sum())) for k, p in module.named_parameters()}


def _grads(module: torch.nn.Module) -> dict[str, torch.Tensor]:
    return {f"grad.{k}": p.grad.float() for k, p in module.named_parameters() if p.grad is not None}


def column_fixture() -> None:
    g = torch.Generator().manual_seed(SEED)
    col = Column(SHAPE, g).to(F64)
    sums = _param_sums(col)
    b, n, m, t_max = 2, 40, 5, 2
    d, h, hkv, dk = SHAPE.d, SHAPE.heads, SHAPE.kv_heads, SHAPE.head_dim
    gi = torch.Generator().manual_seed(SEED + 1)
    x = _bf16(torch.randn(b, n, d, generator=gi, dtype=F64))
    start = 3
    pos = (torch.arange(n) + start + m).expand(b, n).contiguous()
    h1 = (0.3 * torch.randn(b, h, dk, dk, generator=gi, dtype=F64)).float().to(F64)
    ck = _bf16(torch.randn(b, m, hkv, dk, generator=gi, dtype=F64))
    cv = _bf16(torch.randn(b, m, hkv, dk, generator=gi, dtype=F64))
    cpos = (torch.arange(m) + start).expand(b, m).contiguous()
    hist = _bf16(torch.randn(b, SHAPE.key_history, d, generator=gi, dtype=F64))
    active = torch.rand(b, n, generator=gi) < 0.7
    rec_z = _bf16(torch.randn(b, n, d, generator=gi, dtype=F64))
    rec_k = _bf16(normalize_keys(torch.randn(b, n, h, dk, generator=gi, dtype=F64)))
    rec_v = _bf16(torch.randn(b, n, h, dk, generator=gi, dtype=F64))
    rec_beta = _bf16(torch.sigmoid(torch.randn(b, n, h, generator=gi, dtype=F64)))
    attn_k = _bf16(torch.randn(b, n, hkv, dk, generator=gi, dtype=F64))
    attn_v = _bf16(torch.randn(b, n, hkv, dk, generator=gi, dtype=F64))
    up = torch.randn(b, n, d, generator=gi, dtype=F64).float().to(F64) * active[..., None]
    up_h = torch.randn(b, h, dk, dk, generator=gi, dtype=F64).float().to(F64)

    leaves = {k: t.clone().requires_grad_() for k, t in dict(
        x=x, h1=h1, ck=ck, cv=cv, hist=hist, rec_z=rec_z, rec_k=rec_k, rec_v=rec_v, rec_beta=rec_beta,
        attn_k=attn_k, attn_v=attn_v).items()}  # fmt: skip
    zeros_h = torch.zeros(b, h, dk, dk, dtype=F64)
    empty = KVCache(torch.zeros(b, 0, hkv, dk, dtype=F64), torch.zeros(b, 0, hkv, dk, dtype=F64),
                    torch.zeros(b, 0, dtype=torch.long), SHAPE.window)  # fmt: skip
    state = ColumnState(
        h=(zeros_h, leaves["h1"]),
        kv=(empty, KVCache(leaves["ck"], leaves["cv"], cpos, SHAPE.window)),
        key_history=(torch.zeros(b, SHAPE.key_history, d, dtype=F64), leaves["hist"]),
    )
    proj = Projections(leaves["rec_z"], leaves["rec_k"], leaves["rec_v"], leaves["rec_beta"], leaves["attn_k"],
                       leaves["attn_v"])  # fmt: skip
    y, new, written = col.step(leaves["x"], pos, state, 1, carry=Carry(active, proj))
    ((y * up).sum() + (new.h[1] * up_h).sum()).backward()
    _save(
        "column_step", x=x.float(), pos=pos, h1=h1.float(), ck=ck.float(), cv=cv.float(), cpos=cpos,
        hist=hist.float(), active=active, rec_z=rec_z.float(), rec_k=rec_k.float(), rec_v=rec_v.float(),
        rec_beta=rec_beta.float(), attn_k=attn_k.float(), attn_v=attn_v.float(), up=up.float(), up_h=up_h.float(),
        t_max=t_max, y=y, h_new=new.h[1], hist_next=new.key_history[1], kv_k=new.kv[1].k, kv_v=new.kv[1].v,
        kv_pos=new.kv[1].pos, w_z=written.rec_z, w_k=written.rec_k, w_v=written.rec_v, w_beta=written.rec_beta,
        w_ak=written.attn_k, w_av=written.attn_v,
        **{f"dleaf.{k}": t.grad for k, t in leaves.items()}, **_grads(col), **sums,
    )  # fmt: skip


def _loop(columns: int, t_max: int, b_h: float, w_scale: float) -> tuple[Loop, dict[str, np.ndarray]]:
    g = torch.Generator().manual_seed(SEED)
    cols = [Column(SHAPE, g) for _ in range(columns)]
    loop = Loop(cols, HaltingHead(SHAPE.d, g), SHAPE.d, t_max, 0.01)
    sums = _param_sums(loop)  # before the bias is set: the seed's own draws
    with torch.no_grad():
        loop.halting_head().b_h.fill_(b_h)
        loop.halting_head().w_h.mul_(w_scale)  # a wider logit spread: exits at every pass
        loop.u.copy_(0.5 * torch.randn(t_max, SHAPE.d, generator=torch.Generator().manual_seed(SEED + 2)))
    return loop.to(F64), sums


def _cold(b: int, t_max: int, columns: int) -> list[ColumnState]:
    d, hkv, dk = SHAPE.d, SHAPE.kv_heads, SHAPE.head_dim
    out = []
    for _ in range(columns):
        out.append(ColumnState(
            h=tuple(torch.zeros(b, SHAPE.heads, dk, dk, dtype=F64) for _ in range(t_max)),
            kv=tuple(KVCache(torch.zeros(b, 0, hkv, dk, dtype=F64), torch.zeros(b, 0, hkv, dk, dtype=F64),
                             torch.zeros(b, 0, dtype=torch.long), SHAPE.window) for _ in range(t_max)),
            key_history=tuple(torch.zeros(b, SHAPE.key_history, d, dtype=F64) for _ in range(t_max)),
        ))  # fmt: skip
    return out


def loop_fixtures() -> None:
    columns, t_max, b, n = 2, 3, 2, 48
    for name, rule_kind, b_h, w_scale in (("loop_act", "act", 1.0, 4.0), ("loop_cdf", "cdf", 0.0, 1.0)):
        loop, sums = _loop(columns, t_max, b_h, w_scale)
        gi = torch.Generator().manual_seed(SEED + 3)
        x0 = _bf16(torch.randn(b, n, SHAPE.d, generator=gi, dtype=F64)).requires_grad_()
        pos = torch.arange(n).expand(b, n).contiguous()
        up = torch.randn(b, n, SHAPE.d, generator=gi, dtype=F64).float().to(F64)
        rule = CdfRule(loop.halting_head(), 0.5) if rule_kind == "cdf" else None
        res = loop.forward(x0, pos, _cold(b, t_max, columns), exit_rule=rule)
        ((res.y * up).sum() + 0.1 * res.ponder.sum()).backward()
        # the decisions' margins, recomputed from the pass outputs with the reference's own head
        head, eps = loop.halting_head(), loop.halt_epsilon
        with torch.no_grad():
            margins = []
            if rule_kind == "act":
                cum = torch.zeros(b, n, dtype=F64)
                for t in range(t_max - 1):
                    p = head.probability(res.per_pass[t], t)
                    margins.append(cum + p - (1.0 - eps))
                    cum = cum + p
            else:
                from vesper.exits import cdf_advance, cdf_begin, hazard_baseline  # noqa: PLC0415

                base = hazard_baseline(t_max)
                surv, cdf = cdf_begin(res.n_iters)
                for t in range(t_max - 1):
                    surv, cdf = cdf_advance(head.logit(res.per_pass[t], t).double() + base[t], surv, cdf)
                    margins.append(cdf - 0.5)
            active_before = torch.stack([res.n_iters > t for t in range(t_max - 1)])
            mg = torch.stack(margins)
            live = mg[active_before]
            print(name, "n_iters histogram", torch.bincount(res.n_iters.flatten()).tolist(),
                  "min |margin|", float(live.abs().min()))  # fmt: skip
        _save(
            name, x0=x0.detach().float(), pos=pos, up=up.float(), b_h=b_h, u=loop.u.detach(), t_max=t_max,
            columns=columns, rule=rule_kind, w_scale=w_scale, y=res.y, n_iters=res.n_iters, ponder=res.ponder,
            per_pass=res.per_pass.float(), margins=mg, dx0=x0.grad, **_grads(loop), **sums,
        )  # fmt: skip


# config 4's looped model: d=512, 8 heads x 64, kv_groups 4, window 512,
# relu^2 FFN of 3 x d, block 64, key filter of 4 taps, 13 columns, 8 passes, ACT with epsilon 0.01
# and the random-init halting head, vocabulary 32000; reduced to B x T = 2 x 96 tokens so the float64
# reference runs on a CPU in about a minute
C4_SHAPE = ColumnShape(d=512, heads=8, kv_groups=4, head_dim=64, window=512, rotary_base=10000.0, ffn_mult=3,
                       block=64, key_conv=4)  # fmt: skip
C4_COLUMNS, C4_TMAX, C4_VOCAB, C4_B, C4_N, C4_SEED = 13, 8, 32000, 2, 128, 0


def config4_fixture() -> None:
    """The config-4 model's pass counts: embedding, 13 columns and the halting head drawn in the
    model's order from seed 0 (``vesper/model.py:49-56``), token ids uniform over the vocabulary."""
    g = torch.Generator().manual_seed(C4_SEED)
    emb = TiedEmbedding(C4_VOCAB, C4_SHAPE.d, g)
    cols = [Column(C4_SHAPE, g) for _ in range(C4_COLUMNS)]
    loop = Loop(cols, HaltingHead(C4_SHAPE.d, g), C4_SHAPE.d, C4_TMAX, 0.01)
    sums = {**{f"sum.embedding.{k}": v for k, v in ((k[4:], v) for k, v in _param_sums(emb).items())},
            **_param_sums(loop)}  # fmt: skip
    emb, loop = emb.to(F64), loop.to(F64)
    tokens = torch.randint(0, C4_VOCAB, (C4_B, C4_N), generator=torch.Generator().manual_seed(C4_SEED + 1))
    pos = torch.arange(C4_N).expand(C4_B, C4_N).contiguous()
    d, hkv, dk = C4_SHAPE.d, C4_SHAPE.kv_heads, C4_SHAPE.head_dim
    states = [ColumnState(
        h=tuple(torch.zeros(C4_B, C4_SHAPE.heads, dk, dk, dtype=F64) for _ in range(C4_TMAX)),
        kv=tuple(KVCache(torch.zeros(C4_B, 0, hkv, dk, dtype=F64), torch.zeros(C4_B, 0, hkv, dk, dtype=F64),
                         torch.zeros(C4_B, 0, dtype=torch.long), C4_SHAPE.window) for _ in range(C4_TMAX)),
        key_history=tuple(torch.zeros(C4_B, C4_SHAPE.key_history, d, dtype=F64) for _ in range(C4_TMAX)),
    ) for _ in range(C4_COLUMNS)]  # fmt: skip
    with torch.no_grad():
        res = loop.forward(emb.embed(tokens), pos, states)
        head, eps = loop.halting_head(), loop.halt_epsilon
        cum = torch.zeros(C4_B, C4_N, dtype=F64)
        margins = []
        for t in range(C4_TMAX - 1):
            p = head.probability(res.per_pass[t], t)
            margins.append(cum + p - (1.0 - eps))
            cum = cum + p
        mg = torch.stack(margins)
        live = mg[torch.stack([res.n_iters > t for t in range(C4_TMAX - 1)])]
        print("config4 n_iters histogram", torch.bincount(res.n_iters.flatten(), minlength=C4_TMAX + 1).tolist(),
              "min |margin|", float(live.abs().min()))  # fmt: skip
    _save("loop_config4", tokens=tokens, pos=pos, n_iters=res.n_iters, margins=mg, y=res.y.float(), ponder=res.ponder,
          **sums)  # fmt: skip


def decode_fixture() -> None:
    """The reference's one-token decoding (``vesper/decode.py:29-46`` ``decode_step``: the loop at a
    fixed depth under ``DenseRule`` over ``RingKVCache`` windows, the head on the token) fed two
    rows token by token: each row's prompt, then its greedy continuation. Float64 on the CPU; the
    embedding, columns, halting head and output norm drawn in the model's order from the seed."""
    from vesper.column import RMSNorm as RefRMSNorm  # noqa: PLC0415
    from vesper.column import init_column_state  # noqa: PLC0415
    from vesper.loop import DenseRule  # noqa: PLC0415

    columns, t_max, vocab, depth, prompt, gen = 2, 3, 256, 2, 24, 8
    g = torch.Generator().manual_seed(SEED)
    emb = TiedEmbedding(vocab, SHAPE.d, g)
    cols = [Column(SHAPE, g) for _ in range(columns)]
    loop = Loop(cols, HaltingHead(SHAPE.d, g), SHAPE.d, t_max, 0.01)
    norm_out = RefRMSNorm(SHAPE.d)
    sums = {**{f"sum.embedding.{k[4:]}": v for k, v in _param_sums(emb).items()}, **_param_sums(loop)}
    with torch.no_grad():
        loop.u.copy_(0.5 * torch.randn(t_max, SHAPE.d, generator=torch.Generator().manual_seed(SEED + 2)))
    emb, loop, norm_out = emb.to(F64), loop.to(F64), norm_out.to(F64)
    prompts = torch.randint(0, vocab, (2, prompt), generator=torch.Generator().manual_seed(SEED + 4))
    logits_all, ids_all = [], []
    with torch.no_grad():
        for row in range(2):
            states = [init_column_state(SHAPE, 1, t_max, F64, torch.device("cpu"), ring=True) for _ in range(columns)]
            seq = prompts[row].tolist()
            row_logits = []
            for i in range(prompt + gen):
                token = torch.tensor([[seq[i]]])
                res = loop.forward(emb.embed(token), torch.tensor([[i]]), states, passes=depth,
                                   exit_rule=DenseRule())  # fmt: skip
                states = list(res.states)
                logits = emb.logits(norm_out.forward(res.y[:, -1:]))[0, 0]
                row_logits.append(logits)
                if i + 1 >= prompt and len(seq) < prompt + gen:
                    seq.append(int(logits.argmax()))
            logits_all.append(torch.stack(row_logits))
            ids_all.append(torch.tensor(seq))
    print("decode fixture generated", [t[prompt:].tolist() for t in ids_all])
    _save("decode_greedy", tokens=torch.stack(ids_all), logits=torch.stack(logits_all), prompt=prompt, gen=gen,
          depth=depth, vocab=vocab, columns=columns, t_max=t_max, u=loop.u.detach(), **sums)  # fmt: skip


if __name__ == "__main__":
    torch.manual_seed(0)
    which = set(sys.argv[1:]) or {"column", "loop", "config4", "decode"}
    if "column" in which:
        column_fixture()
    if "loop" in which:
        loop_fixtures()
    if "config4" in which:
        config4_fixture()
    if "decode" in which:
        decode_fixture()
