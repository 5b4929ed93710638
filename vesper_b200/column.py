"""One column on a B200 (the contract of ``vesper/column.py`` of mstampfli/vesper-preview).

Pre-RMSNorm residual sublayers in the reference's order: the recurrent core (projections, causal
key filter, delta-rule scan), windowed attention, the feed-forward ``W_2 relu(W_1 x)^2``. The
classes keep the reference's parameter names, shapes and initialization draws, so a reference
``state_dict`` loads unchanged, and its per-pass state (``ColumnState``), its copy-forward
(``Carry`` / ``Projections``) and its ``step`` contract. What runs differs: RMSNorm, the key filter,
the scan (which forms the write strength ``sigmoid(W_beta x)`` inside its kernels, so the carried
``rec_beta`` holds logits) and the attention are this package's sm_100a kernels (no reference
scan: the reference's ``delta_scan_chunked`` is the oracle the tests compare with), the
copy-forward merges are one
multi-tensor select per merge point, and with a carry the attention computes the active queries
only (the halted ones' outputs are discarded by the loop anyway). Projections stay cuBLAS GEMMs.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Literal

import torch
import torch.nn.functional as F  # noqa: N812
from torch import Tensor, nn

from vesper_b200.attention import KVCache, RingKVCache, WindowedAttention, kv_cache_empty, kv_ring_empty
from vesper_b200.contracts import ContractError, Dims, check_shape
from vesper_b200.kernels.act import relu_square, residual_add
from vesper_b200.kernels.compact import Compaction, compact_index, expand_rows, gather_rows, select_rows
from vesper_b200.kernels.delta_scan import (
    delta_scan_fused,
    delta_scan_fused_fp32,
    delta_scan_step_,
    fused_scan_available,
)
from vesper_b200.kernels.keys import fused_keys
from vesper_b200.kernels.norm import add_rms_norm, fused_rms_norm
from vesper_b200.kernels.rotary import inv_freq
from vesper_b200.kernels.slabs import slab_ffn, slab_linears, slab_residual_norm

ScanImpl = Literal["fused", "fused-fp32"]
SCAN_IMPLS: tuple[ScanImpl, ...] = ("fused", "fused-fp32")
FUSED_INPUT_DTYPES: dict[ScanImpl, torch.dtype] = {"fused": torch.bfloat16, "fused-fp32": torch.float32}
STATE_DTYPE = torch.float32
RMS_EPS = 1e-6  # inside the root (vesper/column.py:59)
RMS_SCALE_FLOOR = 1e-3  # the row scale's floor (vesper/column.py:60)


@dataclass(frozen=True)
class ColumnShape:
    """The column's geometry (``vesper/column.py:64-90``)."""

    d: int
    heads: int
    kv_groups: int
    head_dim: int
    window: int
    rotary_base: float
    ffn_mult: int
    block: int
    key_conv: int

    @property
    def key_history(self) -> int:
        return max(self.key_conv - 1, 0)

    @property
    def kv_heads(self) -> int:
        return self.heads // self.kv_groups


@dataclass(frozen=True)
class Projections:
    """What a chunk writes into a pass's states per position (``vesper/column.py:122-137``).

    ``rec_beta`` holds the write-strength LOGITS ``W_beta x`` here, not ``beta``: the scan forms
    ``beta = sigmoid(logits)`` inside its kernels (``from_logits``), so a halted token's carried
    write strength is carried as the logits it was computed from (the same ``beta`` results).
    """

    rec_z: Tensor
    rec_k: Tensor
    rec_v: Tensor
    rec_beta: Tensor
    attn_k: Tensor
    attn_v: Tensor


@dataclass(frozen=True)
class Carry:
    """Which tokens are active (``bool[b, n]``) and what the halted ones write instead; ``rows``
    (optional, ``compact_flat(active, ...)``) lets the feed-forward block run on the active rows
    only."""

    active: Tensor
    projections: Projections
    rows: Compaction | None = None


@dataclass(frozen=True)
class ColumnState:
    """Per-pass recurrent states ``h[t] [b,h,dk,dk]``, windows ``kv[t]``, key histories
    ``key_history[t] [b,K-1,d]`` (``vesper/column.py:429-441``)."""

    h: tuple[Tensor, ...]
    kv: tuple[KVCache | RingKVCache, ...]
    key_history: tuple[Tensor, ...]


def init_column_state(shape: ColumnShape, b: int, t_max: int, dtype: torch.dtype, device: torch.device, *,
                      ring: bool = False) -> ColumnState:  # fmt: skip
    """Cold state (``vesper/column.py:444-480``): zero states and histories in
    ``promote_types(dtype, float32)``, empty windows in ``dtype`` (``ring``: unwritten rings for
    one-token decoding)."""
    if t_max < 1:
        msg = f"t_max must be at least 1, got {t_max}"
        raise ValueError(msg)
    dk = shape.head_dim
    sdt = torch.promote_types(dtype, torch.float32)
    empty = kv_ring_empty if ring else kv_cache_empty
    return ColumnState(
        h=tuple(torch.zeros(b, shape.heads, dk, dk, dtype=sdt, device=device) for _ in range(t_max)),
        kv=tuple(empty(b, shape.kv_heads, dk, shape.window, dtype, device) for _ in range(t_max)),
        key_history=tuple(torch.zeros(b, shape.key_history, shape.d, dtype=sdt, device=device) for _ in range(t_max)),
    )


def map_state(state: ColumnState, f: Callable[[Tensor], Tensor]) -> ColumnState:
    """Every tensor of ``state`` through ``f`` in a fixed order (``vesper/column.py:500-517``)."""

    def window(c: KVCache | RingKVCache) -> KVCache | RingKVCache:
        if isinstance(c, RingKVCache):
            return RingKVCache(k=f(c.k), v=f(c.v), pos=f(c.pos), valid=f(c.valid), window=c.window)
        return KVCache(k=f(c.k), v=f(c.v), pos=f(c.pos), window=c.window)

    return ColumnState(
        h=tuple(f(h) for h in state.h),
        kv=tuple(window(c) for c in state.kv),
        key_history=tuple(f(z) for z in state.key_history),
    )


def state_tensors(states: Sequence[ColumnState]) -> list[Tensor]:
    """Every tensor of ``states`` as a flat list in ``map_state``'s order (for captured graphs)."""
    out: list[Tensor] = []
    for state in states:
        map_state(state, lambda t: out.append(t) or t)
    return out


def with_state_tensors(templates: Sequence[ColumnState], tensors: Sequence[Tensor]) -> list[ColumnState]:
    """The inverse of ``state_tensors``."""
    if len(state_tensors(templates)) != len(tensors):
        msg = f"{len(tensors)} state tensors for a structure of {len(state_tensors(templates))}"
        raise ValueError(msg)
    feed = iter(tensors)
    return [map_state(s, lambda _: next(feed)) for s in templates]


def _require_cuda(x: Tensor, what: str) -> None:
    if x.device.type != "cuda":
        msg = f"the {what} runs on CUDA only, got {x.device}"
        raise ContractError(msg)


class RMSNorm(nn.Module):
    """``x / sqrt(mean(x^2) + 1e-6) * g``, scale-safe, one kernel each way (``fused_rms_norm``).

    Every consumer of a norm's output in the column, the halting head and the output head is a
    matrix product, which autocast runs in its lower dtype, casting its float32 input each time.
    Under CUDA autocast the kernel therefore rounds its float32 result to the autocast dtype as it
    stores it (and its backward reads that dtype's gradient): the same rounding as a cast, so the
    same values and gradients, with no float32 output and no cast kernels either way.
    """

    def __init__(self, d: int) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(d))

    def forward(self, x: Tensor) -> Tensor:
        d = self.weight.shape[0]
        if x.shape[-1] != d:
            msg = f"RMSNorm: last axis must be {d}, got {x.shape[-1]} (shape {tuple(x.shape)})"
            raise ContractError(msg)
        return fused_rms_norm(x, self.weight, RMS_SCALE_FLOOR, RMS_EPS, self._out_dtype(x))

    def add_forward(self, x: Tensor, r: Tensor) -> tuple[Tensor, Tensor]:
        """``(x + r, forward(x + r))``: the residual add and this norm of its sum, one kernel each
        way over a float32 residual stream (the same values and gradients as the two steps)."""
        d = self.weight.shape[0]
        if x.shape[-1] != d:
            msg = f"RMSNorm: last axis must be {d}, got {x.shape[-1]} (shape {tuple(x.shape)})"
            raise ContractError(msg)
        return add_rms_norm(x, r, self.weight, RMS_SCALE_FLOOR, RMS_EPS, self._out_dtype(x))

    @staticmethod
    def _out_dtype(x: Tensor) -> torch.dtype | None:
        """The autocast dtype for a float32 input under CUDA autocast (rounded inside the kernel,
        no cast kernels), else None (the input's dtype)."""
        if x.dtype == torch.float32 and x.is_cuda and torch.is_autocast_enabled("cuda"):
            return torch.get_autocast_dtype("cuda")
        return None


class RecurrentSublayer(nn.Module):
    """``q, k, v``, the write strength, the causal key filter, the delta-rule scan, ``W_o``."""

    def __init__(self, shape: ColumnShape, generator: torch.Generator | None = None) -> None:
        """The reference's parameters and draws (``vesper/column.py:198-234``)."""
        super().__init__()
        d, heads, head_dim = shape.d, shape.heads, shape.head_dim
        if heads * head_dim != d:
            msg = f"heads ({heads}) * head_dim ({head_dim}) must equal d ({d})"
            raise ValueError(msg)
        if shape.block < 1:
            msg = f"block must be at least 1, got {shape.block}"
            raise ValueError(msg)
        self.heads, self.head_dim, self.block = heads, head_dim, shape.block
        self.scan_impl: ScanImpl = "fused"
        std = 1.0 / math.sqrt(d)
        self.w_q = nn.Parameter(torch.randn(d, d, generator=generator) * std)
        self.w_k = nn.Parameter(torch.randn(d, d, generator=generator) * std)
        self.w_v = nn.Parameter(torch.randn(d, d, generator=generator) * std)
        self.w_o = nn.Parameter(torch.randn(d, d, generator=generator) * std)
        self.w_beta = nn.Parameter(torch.randn(heads, d, generator=generator) * std)
        self.key_conv = shape.key_conv
        self.conv_k: nn.Parameter | None = None
        if shape.key_conv:
            bound = 1.0 / math.sqrt(shape.key_conv)
            self.conv_k = nn.Parameter(torch.rand(shape.key_conv, d, generator=generator) * (2 * bound) - bound)

    def project_logits(self, x: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor]:
        """``q, v [b,n,h,dk]``, the key input ``z = W_k x [b,n,d]`` and the write-strength logits
        ``W_beta x [b,n,h]``, which the scan turns into ``beta`` inside its kernels."""
        dims: Dims = {}
        check_shape("x", x, ("b", "n", "d"), dims)
        b, n = dims["b"], dims["n"]
        q = F.linear(x, self.w_q).view(b, n, self.heads, self.head_dim)
        z = F.linear(x, self.w_k)
        v = F.linear(x, self.w_v).view(b, n, self.heads, self.head_dim)
        return q, z, v, F.linear(x, self.w_beta)

    def project(self, x: Tensor) -> tuple[Tensor, Tensor, Tensor, Tensor]:
        """``q, v [b,n,h,dk]``, ``z = W_k x [b,n,d]`` and ``beta = sigmoid(W_beta x)``
        (``vesper/column.py:236-253``); the column itself uses ``project_logits``."""
        q, z, v, logits = self.project_logits(x)
        return q, z, v, torch.sigmoid(logits)

    def keys(self, z: Tensor, history: Tensor) -> tuple[Tensor, Tensor]:
        """Normalized keys from the filter over ``(history, z)`` and the next history
        (``vesper/column.py:255-289``): the newest ``K-1`` inputs, an owned float32 copy."""
        b, n, d = z.shape
        if n == 0:
            return z.view(b, 0, self.heads, self.head_dim), history
        if self.conv_k is None:  # no filter: the key is normalize_keys(z), a one-tap filter of one
            taps = torch.ones(1, d, dtype=torch.float32, device=z.device)
            return fused_keys(z, history, taps, self.heads), history
        width = self.key_conv
        k = fused_keys(z, history, self.conv_k, self.heads)
        compute = torch.promote_types(z.dtype, torch.float32)
        tail = z[:, max(0, n - (width - 1)) :].to(compute)
        return k, torch.cat([history.to(compute)[:, n:], tail], dim=1)

    def scan(self, q: Tensor, k: Tensor, v: Tensor, beta: Tensor, state: Tensor, *,
             from_logits: bool = False) -> tuple[Tensor, Tensor]:  # fmt: skip
        """The scan (``scan_impl``) with autocast off, then ``W_o`` in the activation dtype;
        ``from_logits``: ``beta`` holds the write-strength logits (the kernels form the sigmoid)."""
        o, new_state = self.scan_outputs(q, k, v, beta, state, from_logits=from_logits)
        return F.linear(o.flatten(2), self.w_o), new_state

    def scan_outputs(self, q: Tensor, k: Tensor, v: Tensor, beta: Tensor, state: Tensor, *,
                     from_logits: bool = False) -> tuple[Tensor, Tensor]:  # fmt: skip
        """The scan's outputs ``o [b,n,h,dk]`` in ``q``'s dtype (before ``W_o``) and new state."""
        kernel = delta_scan_fused if self.scan_impl == "fused" else delta_scan_fused_fp32
        dtype = FUSED_INPUT_DTYPES[self.scan_impl]
        with torch.autocast(device_type=q.device.type, enabled=False):
            o, new_state = kernel(q.to(dtype), k.to(dtype), v.to(dtype), beta.to(dtype), state.to(STATE_DTYPE),
                                  from_logits=from_logits)  # fmt: skip
        return o.to(q.dtype), new_state

    def forward(self, x: Tensor, state: Tensor, history: Tensor) -> tuple[Tensor, Tensor, Tensor]:
        q, z, v, logits = self.project_logits(x)
        k, history_next = self.keys(z, history)
        y, state_next = self.scan(q, k, v, logits, state, from_logits=True)
        return y, state_next, history_next


class FFN(nn.Module):
    """``W_2 relu(W_1 x)^2`` (``vesper/ffn.py:20-60``), the squared ReLU as one kernel each way
    with the reference's arithmetic (``vesper_b200.kernels.act.relu_square``)."""

    def __init__(self, d: int, ffn_mult: int, generator: torch.Generator | None = None) -> None:
        super().__init__()
        if ffn_mult < 1:
            msg = f"ffn_mult must be at least 1, got {ffn_mult}"
            raise ValueError(msg)
        hidden = ffn_mult * d
        self.w1 = nn.Parameter(torch.randn(hidden, d, generator=generator) / math.sqrt(d))
        self.w2 = nn.Parameter(torch.randn(d, hidden, generator=generator) / math.sqrt(hidden))

    def forward(self, x: Tensor) -> Tensor:
        return F.linear(relu_square(F.linear(x, self.w1)), self.w2)


def set_scan(model: nn.Module, impl: str) -> int:
    """Choose the scan of every ``RecurrentSublayer`` (``vesper/column.py:353-384``); the
    reference scan is not part of this build (it is the tests' oracle)."""
    if impl not in SCAN_IMPLS:
        msg = f"scan must be one of {SCAN_IMPLS}, got {impl!r}"
        raise ValueError(msg)
    sublayers = [m for m in model.modules() if isinstance(m, RecurrentSublayer)]
    if not sublayers:
        msg = "the model has no recurrent sublayer to set"
        raise ValueError(msg)
    if any(p.device.type != "cuda" for p in model.parameters()):
        msg = "the fused scan needs the model on CUDA"
        raise ValueError(msg)
    if not fused_scan_available():
        msg = "the fused scan needs a CUDA device and the built library"
        raise ValueError(msg)
    for s in sublayers:
        s.scan_impl = impl  # type: ignore[assignment]
    return len(sublayers)


class Column(nn.Module):
    """Recurrent core, windowed attention and FFN, each pre-RMSNorm with a residual."""

    def __init__(self, shape: ColumnShape, generator: torch.Generator | None = None) -> None:
        super().__init__()
        self.norm_rec = RMSNorm(shape.d)
        self.rec = RecurrentSublayer(shape, generator)
        self.norm_attn = RMSNorm(shape.d)
        self.attn = WindowedAttention(shape.d, shape.heads, shape.kv_groups, shape.head_dim, shape.window,
                                      shape.rotary_base, generator)  # fmt: skip
        self.norm_ffn = RMSNorm(shape.d)
        self.ffn = FFN(shape.d, shape.ffn_mult, generator)

    def step(self, x: Tensor, pos: Tensor, state: ColumnState, pass_index: int, *,
             carry: Carry | None = None, zero_halted: bool = False) -> tuple[Tensor, ColumnState, Projections]:  # fmt: skip
        """One pass over a chunk through the state of pass ``pass_index`` (``vesper/column.py:709-812``).

        With a carry, halted tokens write their carried projections: the key input is merged
        before the filter and ``k, v, beta`` after it (one select launch), the attention keys and
        values after their projection (one launch), and the attention runs the active queries
        only. The output at halted positions is not meaningful; the loop discards it.
        ``zero_halted`` (the loop's own use, with a carry) sets those positions to zero in the
        column's last residual add, which the loop would otherwise do in a separate pass.
        """
        if not len(state.h) == len(state.kv) == len(state.key_history):
            msg = f"state has {len(state.h)} recurrent states, {len(state.kv)} windows and {len(state.key_history)} key histories"
            raise ValueError(msg)
        if not 0 <= pass_index < len(state.h):
            msg = f"pass_index must lie in [0, {len(state.h)}), got {pass_index}"
            raise ValueError(msg)
        _require_cuda(x, "column")
        history = state.key_history[pass_index]
        check_shape("state.key_history", history, ("b", "w", "d"),
                    {"b": x.shape[0], "w": max(self.rec.key_conv - 1, 0), "d": x.shape[2]})  # fmt: skip
        if carry is not None:
            dims: Dims = {"b": x.shape[0], "n": x.shape[1], "d": x.shape[2], "h": self.rec.heads,
                          "hkv": self.attn.kv_heads, "dk": self.rec.head_dim}  # fmt: skip
            p = carry.projections
            check_shape("carry.active", carry.active, ("b", "n"), dims, dtype=torch.bool)
            check_shape("carry.rec_z", p.rec_z, ("b", "n", "d"), dims)
            check_shape("carry.rec_k", p.rec_k, ("b", "n", "h", "dk"), dims)
            check_shape("carry.rec_v", p.rec_v, ("b", "n", "h", "dk"), dims)
            check_shape("carry.rec_beta", p.rec_beta, ("b", "n", "h"), dims)
            check_shape("carry.attn_k", p.attn_k, ("b", "n", "hkv", "dk"), dims)
            check_shape("carry.attn_v", p.attn_v, ("b", "n", "hkv", "dk"), dims)

        window = state.kv[pass_index]
        if carry is not None and carry.rows is not None:  # every per-token step on the active rows only
            x, h_new, history_next, kv_new, written = self._step_rows(x, pos, state.h[pass_index], history,
                                                                      window, carry)  # fmt: skip
        else:
            q, z, v, beta = self.rec.project_logits(self.norm_rec.forward(x))  # beta: the logits
            if carry is not None:
                (z,) = select_rows(carry.active, [z], [carry.projections.rec_z.to(z.dtype)])
            k, history_next = self.rec.keys(z, history)
            if carry is not None:
                p = carry.projections
                k, v, beta = select_rows(carry.active, [k, v, beta],
                                         [p.rec_k.to(k.dtype), p.rec_v.to(v.dtype), p.rec_beta.to(beta.dtype)])  # fmt: skip
            r, h_new = self.rec.scan(q, k, v, beta, state.h[pass_index], from_logits=True)
            x, xn = self.norm_attn.add_forward(x, r)  # x + r and norm_attn of it, one kernel

            aq, ak, av = self.attn.project(xn, pos)
            compaction = None
            if carry is not None:
                ak, av = select_rows(carry.active, [ak, av],
                                     [carry.projections.attn_k.to(ak.dtype), carry.projections.attn_v.to(av.dtype)])  # fmt: skip
                compaction = compact_index(carry.active, qpos_offset=window.k.shape[1])
            a, kv_new = self.attn.attend(aq, ak, av, pos, window, compaction)
            x, xn = self.norm_ffn.add_forward(x, a)  # x + a and norm_ffn of it, one kernel
            keep = carry.active if zero_halted and carry is not None else None
            x = residual_add(x, self.ffn.forward(xn), keep)  # the halted rows zeroed here when asked
            written = Projections(rec_z=z, rec_k=k, rec_v=v, rec_beta=beta, attn_k=ak, attn_v=av)
        h = tuple(h_new if i == pass_index else s for i, s in enumerate(state.h))
        kv = tuple(kv_new if i == pass_index else c for i, c in enumerate(state.kv))
        hist = tuple(history_next if i == pass_index else o for i, o in enumerate(state.key_history))
        return x, ColumnState(h=h, kv=kv, key_history=hist), written

    def _step_rows(self, x: Tensor, pos: Tensor, h: Tensor, history: Tensor, window: KVCache,
                   carry: Carry) -> tuple[Tensor, Tensor, Tensor, KVCache, Projections]:  # fmt: skip
        """``step`` with a carry whose ``rows`` compact the active tokens: every per-token step runs
        on those rows only (bucketed on their live count, ``vesper_b200.kernels.slabs``), the
        residual stream stays compact from the input to the output, and only the key filter, the
        scan and the attention's keys and values see every token (the halted ones' carried
        projections in place). The output is zero at the halted tokens, as the loop leaves them.
        Returns the output, the new state, key history and window, and the written projections."""
        rows, p = carry.rows, carry.projections
        assert rows is not None and rows.relayout is not None
        b, n, d = x.shape
        heads, kv_heads, dk = self.attn.heads, self.attn.kv_heads, self.attn.head_dim
        flat, first, count = (1, b * n), rows.slab_first, rows.counts
        dtype = RMSNorm._out_dtype(x) or x.dtype  # the autocast dtype, as F.linear would cast

        # the active rows of the residual stream; compact buffers are used as views [cap, width]
        # (a view's backward is a view; indexing's would zero-fill and copy the whole buffer)
        (xc,) = gather_rows(rows, [x.reshape(*flat, d)])
        xc = xc.view(b * n, d)
        weights = [w.to(dtype) for w in (self.rec.w_q, self.rec.w_k, self.rec.w_v, self.rec.w_beta)]
        qc, zc, vc, bc = slab_linears(xc, weights, count, first,
                                      norm=(self.norm_rec.weight, RMS_SCALE_FLOOR, RMS_EPS))  # fmt: skip
        q, z, v, beta = expand_rows(
            rows, [qc.view(*flat, d), zc.view(*flat, d), vc.view(*flat, d), bc.view(*flat, self.rec.heads)],
            [None, p.rec_z.to(dtype).reshape(*flat, d), p.rec_v.to(dtype).reshape(*flat, d),
             p.rec_beta.to(dtype).reshape(*flat, self.rec.heads)],
        )  # fmt: skip
        q, z = q.view(b, n, self.rec.heads, self.rec.head_dim), z.view(b, n, d)
        v, beta = v.view(b, n, self.rec.heads, self.rec.head_dim), beta.view(b, n, self.rec.heads)
        k, history_next = self.rec.keys(z, history)
        (k,) = select_rows(carry.active, [k], [p.rec_k.to(k.dtype)])
        o, h_new = self.rec.scan_outputs(q, k, v, beta, h, from_logits=True)

        (oc,) = gather_rows(rows, [o.reshape(*flat, d)])
        sc, xnc = slab_residual_norm(xc, oc.view(b * n, d), self.rec.w_o.to(dtype), self.norm_attn.weight, count, first,
                                     RMS_SCALE_FLOOR, RMS_EPS)  # fmt: skip

        with torch.no_grad():
            (pc,) = gather_rows(rows, [pos.reshape(*flat, 1)])  # positions of the compact rows
        weights = [w.to(dtype) for w in (self.attn.w_q, self.attn.w_k, self.attn.w_v)]
        turn = (pc.view(-1), inv_freq(dk, self.attn.rotary_base, x.device), (heads, kv_heads, 0))
        aqc, akc, avc = slab_linears(xnc, weights, count, first, rotary=turn)
        ak, av = expand_rows(rows, [akc.view(*flat, kv_heads * dk), avc.view(*flat, kv_heads * dk)],
                             [p.attn_k.to(dtype).reshape(*flat, kv_heads * dk),
                              p.attn_v.to(dtype).reshape(*flat, kv_heads * dk)])  # fmt: skip
        ak, av = ak.view(b, n, kv_heads, dk), av.view(b, n, kv_heads, dk)
        (aq,) = expand_rows(rows.relayout, [aqc.view(*flat, heads * dk)])  # packed per batch row
        compaction = compact_index(carry.active, qpos_offset=window.k.shape[1])
        oa, kv_new = self.attn.attend_packed(aq.view(b, n, heads, dk), ak, av, pos, window, compaction)
        (oac,) = gather_rows(rows.relayout, [oa.reshape(*flat, heads * dk)])  # per-row packed -> flat
        sc, xnc = slab_residual_norm(sc, oac.view(b * n, heads * dk), self.attn.w_o.to(dtype), self.norm_ffn.weight,
                                     count, first, RMS_SCALE_FLOOR, RMS_EPS)  # fmt: skip

        outc = slab_ffn(xnc, self.ffn.w1.to(dtype), self.ffn.w2.to(dtype), count, first, residual=sc)
        (out,) = expand_rows(rows, [outc.view(*flat, d)])  # zero at the halted tokens
        written = Projections(rec_z=z, rec_k=k, rec_v=v, rec_beta=beta, attn_k=ak, attn_v=av)
        return out.view(b, n, d), h_new, history_next, kv_new, written

    def step_decode(self, x: Tensor, pos: Tensor, state: ColumnState, pass_index: int) -> Tensor:
        """One decoding token per row through pass ``pass_index``'s state, updated IN PLACE.

        What ``step`` computes for ``n = 1`` over a ``RingKVCache`` window (``vesper/column.py:
        709-812`` with ``attend_ring``), with every carried buffer updated where it lies so a
        captured decode step needs no copies: the recurrent state by the one-token scan kernel
        (``delta_scan_step_``, the write strength formed from its logits), the key history shifted
        by one, the ring written by the attention kernel. ``x [b, 1, d]``, ``pos [b, 1]``.
        """
        ring = state.kv[pass_index]
        if not isinstance(ring, RingKVCache):
            msg = "step_decode carries a RingKVCache window (init_column_state(..., ring=True))"
            raise ContractError(msg)
        history, h = state.key_history[pass_index], state.h[pass_index]
        q, z, v, logits = self.rec.project_logits(self.norm_rec.forward(x))
        k, _ = self.rec.keys(z, history)
        if history.shape[1]:
            with torch.no_grad():
                history.copy_(torch.cat([history[:, 1:], z.to(history.dtype)], dim=1))
        dtype = FUSED_INPUT_DTYPES[self.rec.scan_impl]
        with torch.autocast(device_type=x.device.type, enabled=False):
            o = delta_scan_step_(q.to(dtype), k.to(dtype), v.to(dtype), logits.to(dtype), h, from_logits=True)
        x = x + F.linear(o.to(q.dtype).flatten(2), self.rec.w_o)
        aq, ak, av = self.attn.project(self.norm_attn.forward(x), pos)
        a, _ = self.attn.attend_ring(aq, ak, av, pos, ring)
        x = x + a
        return x + self.ffn.forward(self.norm_ffn.forward(x))

    def forward(self, x: Tensor, pos: Tensor, state: ColumnState, pass_index: int) -> tuple[Tensor, ColumnState]:
        y, new_state, _ = self.step(x, pos, state, pass_index)
        return y, new_state
