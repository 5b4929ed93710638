"""Generate the golden fixtures of tests/golden/ by running the reference itself.

Run in a container that holds the reference (mstampfli/vesper-preview) source:

    VESPER_REF=<reference checkout> PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py

It imports the reference's own pure-PyTorch modules (``vesper.recurrence``, ``vesper.column``,
``vesper.attention``) and evaluates them in float64 on the CPU with autograd for gradients, on
seeded inputs whose values are exactly representable in bfloat16 (the reference's kernel tests
feed both sides the same bfloat16-valued inputs, ``tests/test_delta_scan_fused.py:47-62``).
Inputs are stored as float32 (lossless for those values) and results as float64. Nothing at test
time reads the reference: the fixtures are the pin.
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

from vesper.attention import WindowedAttention, kv_cache_empty, kv_cache_push  # noqa: E402
from vesper.column import ColumnShape, RecurrentSublayer, RMSNorm  # noqa: E402
from vesper.recurrence import delta_scan_chunked, normalize_keys, write_strength  # noqa: E402

F64 = torch.float64


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(F64)


def _save(name: str, **arrays: torch.Tensor | np.ndarray | int | float) -> None:
    out: dict[str, np.ndarray] = {}
    for key, value in arrays.items():
        if isinstance(value, torch.Tensor):
            value = value.detach().cpu().numpy()
        out[key] = np.asarray(value)
    np.savez_compressed(HERE / f"{name}.npz", **out)


# --- delta scan: tests/test_delta_scan_fused.py SIZES[:4], plus a block-size variant -----------
SCAN_SIZES = [(2, 1, 2, 16), (2, 63, 3, 16), (1, 65, 2, 64), (2, 130, 3, 16)]


def scan_fixtures() -> None:
    for b, n, h, dk in SCAN_SIZES:
        g = torch.Generator().manual_seed(1000 + n)
        q = _bf16(torch.randn(b, n, h, dk, generator=g, dtype=F64))
        k = _bf16(normalize_keys(torch.randn(b, n, h, dk, generator=g, dtype=F64)))
        v = _bf16(torch.randn(b, n, h, dk, generator=g, dtype=F64))
        beta = _bf16(write_strength(torch.randn(b, n, h, generator=g, dtype=F64)))
        h0 = (0.5 * torch.randn(b, h, dk, dk, generator=g, dtype=F64)).float().to(F64)
        d_o = torch.randn(b, n, h, dk, generator=g, dtype=F64).float().to(F64)
        d_s = torch.randn(b, h, dk, dk, generator=g, dtype=F64).float().to(F64)
        ins = [t.clone().requires_grad_() for t in (q, k, v, beta, h0)]
        o, s = delta_scan_chunked(*ins, 64)
        torch.autograd.backward([(o * d_o).sum() + (s * d_s).sum()])
        _save(
            f"scan_{b}x{n}x{h}x{dk}",
            q=q.float(), k=k.float(), v=v.float(), beta=beta.float(), h0=h0.float(),
            d_o=d_o.float(), d_s=d_s.float(), o=o, s=s,
            dq=ins[0].grad, dk=ins[1].grad, dv=ins[2].grad, dbeta=ins[3].grad, dh0=ins[4].grad,
        )  # fmt: skip


# --- key filter: tests/test_keys_fused.py (asymmetric taps, a zero input row) -----------------
KEY_D, KEY_HEADS, KEY_K = 128, 2, 4


def _key_layer() -> RecurrentSublayer:
    shape = ColumnShape(
        d=KEY_D, heads=KEY_HEADS, kv_groups=2, head_dim=KEY_D // KEY_HEADS, window=16,
        rotary_base=10000.0, ffn_mult=2, block=16, key_conv=KEY_K,
    )  # fmt: skip
    layer = RecurrentSublayer(shape, torch.Generator().manual_seed(0)).to(F64)
    with torch.no_grad():
        r = torch.arange(KEY_K, dtype=F64)[:, None]
        j = torch.arange(KEY_D, dtype=F64)[None, :]
        assert layer.conv_k is not None
        layer.conv_k.copy_((r + 1) * 0.5 - 0.003 * j + 0.01 * r * j)
    return layer


def keys_fixtures() -> None:
    for n in (1, 2, 3, 37):
        g = torch.Generator().manual_seed(n)
        z = _bf16(torch.randn(3, n, KEY_D, generator=g, dtype=F64) * 2)
        z[0, 0] = 0.0
        hist = torch.randn(3, KEY_K - 1, KEY_D, generator=g, dtype=F64).float().to(F64)
        up = torch.randn(3, n, KEY_HEADS, KEY_D // KEY_HEADS, generator=g, dtype=F64)
        up = up.float().to(F64)
        layer = _key_layer()
        zs, hs = z.clone().requires_grad_(), hist.clone().requires_grad_()
        k, nxt = layer.keys(zs, hs)
        torch.autograd.backward([(k * up).sum()])
        assert layer.conv_k is not None and layer.conv_k.grad is not None
        _save(
            f"keys_n{n}", z=z.float(), hist=hist.float(), taps=layer.conv_k.detach(),
            up=up.float(), k=k, next_hist=nxt, dz=zs.grad, dtaps=layer.conv_k.grad,
            dhist=hs.grad, heads=KEY_HEADS,
        )  # fmt: skip


# --- RMSNorm: tests/test_norm_fused.py widths and range boundaries ---------------------------
def norm_fixtures() -> None:
    cases: dict[str, tuple[torch.Tensor, torch.Tensor]] = {}
    for width in (512, 384, 33):
        g = torch.Generator().manual_seed(width)
        x = (torch.randn(24, width, generator=g, dtype=F64) * 3).float().to(F64)
        gain = (1 + 0.1 * torch.randn(width, generator=g, dtype=F64)).float().to(F64)
        cases[f"w{width}"] = (x, gain)
    width = 64
    boundary = torch.stack(
        [
            torch.full((width,), 1e20, dtype=F64),
            torch.zeros(width, dtype=F64),
            torch.full((width,), 1e-4, dtype=F64),
            torch.linspace(-1.0, 1.0, width, dtype=F64) * 3e38,
            torch.randn(width, generator=torch.Generator().manual_seed(2), dtype=F64),
        ]
    ).float().to(F64)
    cases["boundary"] = (boundary, torch.ones(width, dtype=F64))
    for name, (x, gain) in cases.items():
        up = torch.randn(x.shape, generator=torch.Generator().manual_seed(1), dtype=F64)
        up = up.float().to(F64)
        norm = RMSNorm(x.shape[-1]).to(F64)
        with torch.no_grad():
            norm.weight.copy_(gain)
        xs = x.clone().requires_grad_()
        y = norm.forward(xs)
        torch.autograd.backward([(y * up).sum()])
        assert xs.grad is not None and norm.weight.grad is not None
        _save(
            f"norm_{name}", x=x.float(), gain=gain.float(), up=up.float(), y=y,
            dx=xs.grad, dg=norm.weight.grad,
        )  # fmt: skip


# --- windowed attention: tests/test_window_attn.py geometry (dk reduced to 16) ----------------
ATT_H, ATT_KV_GROUPS, ATT_DK, ATT_W = 4, 2, 16, 16


def attention_fixtures() -> None:
    hkv = ATT_H // ATT_KV_GROUPS
    d = ATT_H * ATT_DK
    for n, m in ((8, 0), (40, 5), (40, 16)):
        g = torch.Generator().manual_seed(n * 100 + m)
        b, start = 2, 7
        q = _bf16(torch.randn(b, n, ATT_H, ATT_DK, generator=g, dtype=F64))
        k = _bf16(torch.randn(b, n, hkv, ATT_DK, generator=g, dtype=F64))
        v = _bf16(torch.randn(b, n, hkv, ATT_DK, generator=g, dtype=F64))
        pos = (torch.arange(n) + start + m).expand(b, n).contiguous()
        cache = kv_cache_empty(b, hkv, ATT_DK, ATT_W, F64, torch.device("cpu"))
        ck = _bf16(torch.randn(b, m, hkv, ATT_DK, generator=g, dtype=F64))
        cv = _bf16(torch.randn(b, m, hkv, ATT_DK, generator=g, dtype=F64))
        if m > 0:
            cache = kv_cache_push(cache, ck, cv, (torch.arange(m) + start).expand(b, m).contiguous())
        up = torch.randn(b, n, ATT_H, ATT_DK, generator=g, dtype=F64).float().to(F64)
        layer = WindowedAttention(d, ATT_H, ATT_KV_GROUPS, ATT_DK, ATT_W, 10000.0).to(F64)
        with torch.no_grad():
            layer.w_o.copy_(torch.eye(d, dtype=F64))  # the raw attention output, heads merged
        qs, ks, vs = (t.clone().requires_grad_() for t in (q, k, v))
        cks, cvs = ck.clone().requires_grad_(), cv.clone().requires_grad_()
        cache_g = cache
        if m > 0:
            from vesper.attention import KVCache

            cache_g = KVCache(k=cks, v=cvs, pos=cache.pos, window=cache.window)
        y, new = layer.attend(qs, ks, vs, pos, cache_g)
        torch.autograd.backward([(y * up.flatten(2)).sum()])
        _save(
            f"attn_n{n}_m{m}", q=q.float(), k=k.float(), v=v.float(), ck=ck.float(),
            cv=cv.float(), pos=pos, up=up.float(), o=y.view(b, n, ATT_H, ATT_DK),
            dq=qs.grad, dk=ks.grad, dv=vs.grad,
            dck=cks.grad if m > 0 else torch.zeros_like(ck),
            dcv=cvs.grad if m > 0 else torch.zeros_like(cv),
            new_k=new.k, new_pos=new.pos, window=ATT_W,
        )  # fmt: skip


if __name__ == "__main__":
    torch.manual_seed(0)
    scan_fixtures()
    keys_fixtures()
    norm_fixtures()
    attention_fixtures()
    total = sum(p.stat().st_size for p in HERE.glob("*.npz"))
    print(f"wrote {len(list(HERE.glob('*.npz')))} fixtures, {total / 1e6:.2f} MB")
