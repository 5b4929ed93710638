"""Windowed attention sublayer on a B200 (the contract of ``vesper/attention.py`` of
mstampfli/vesper-preview): rotary GQA projections, exact softmax over the last ``window`` keys.

Same parameters (``w_q, w_k, w_v, w_o``), layouts and cache semantics as the reference's
``WindowedAttention`` (``vesper/attention.py:219-407``) and ``KVCache`` / ``kv_cache_push``
(``:30-175``); ``rotary`` (``:178-217``) is one kernel each way (``vesper_b200.kernels.rotary``).
In bfloat16 or float16 the softmax runs in the tcgen05 kernel (``vesper_b200.kernels.window_attn``)
over the cache rows and the chunk directly, in float32 in the same entry points' FFMA kernel (the
reference's float32 mode, its blocked masked softmax, at float32 rounding); given the loop's
compaction of the active tokens, either computes only their queries. One-token decoding carries
a ``RingKVCache`` per pass, attended and written by one batched kernel (``attend_ring``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F  # noqa: N812
from torch import Tensor, nn

from vesper_b200.contracts import ContractError, Dims, check_shape, require
from vesper_b200.kernels.compact import Compaction, expand_rows, gather_rows
from vesper_b200.kernels.rotary import rotary
from vesper_b200.kernels.window_attn import window_attention, window_attention_active

WINDOW_KERNEL_DTYPES = (torch.bfloat16, torch.float16, torch.float32)  # tcgen05 / float32 FFMA kernels


@dataclass(frozen=True, slots=True)
class KVCache:
    """The last ``m <= window`` entries of one window, oldest first: ``k, v [b, m, hkv, dk]``
    (keys rotated) and ``pos [b, m]`` int64."""

    k: Tensor
    v: Tensor
    pos: Tensor
    window: int


def kv_cache_empty(b: int, hkv: int, dk: int, window: int, dtype: torch.dtype, device: torch.device) -> KVCache:
    """An empty cache (``m = 0``) for ``window`` entries (``vesper/attention.py:43-63``)."""
    if window < 1:
        msg = f"window must be at least 1, got {window}"
        raise ValueError(msg)
    return KVCache(
        k=torch.zeros(b, 0, hkv, dk, dtype=dtype, device=device),
        v=torch.zeros(b, 0, hkv, dk, dtype=dtype, device=device),
        pos=torch.zeros(b, 0, dtype=torch.long, device=device),
        window=window,
    )


def kv_cache_push(cache: KVCache, k: Tensor, v: Tensor, pos: Tensor) -> KVCache:
    """The newest ``min(m + n, window)`` entries of the cache followed by the chunk
    (``vesper/attention.py:142-175``); with no new entries, the cache itself."""
    dims: Dims = {}
    check_shape("cache.k", cache.k, ("b", "m", "hkv", "dk"), dims)
    check_shape("cache.v", cache.v, ("b", "m", "hkv", "dk"), dims)
    check_shape("cache.pos", cache.pos, ("b", "m"), dims, dtype=torch.long)
    check_shape("k", k, ("b", "n", "hkv", "dk"), dims)
    check_shape("v", v, ("b", "n", "hkv", "dk"), dims)
    check_shape("pos", pos, ("b", "n"), dims, dtype=torch.long)
    w, m, n = cache.window, dims["m"], dims["n"]
    if n == 0:
        return cache
    keep_new = min(n, w)
    keep_old = min(m, w - keep_new)
    return KVCache(
        k=torch.cat([cache.k[:, m - keep_old :], k[:, n - keep_new :]], dim=1),
        v=torch.cat([cache.v[:, m - keep_old :], v[:, n - keep_new :]], dim=1),
        pos=torch.cat([cache.pos[:, m - keep_old :], pos[:, n - keep_new :]], dim=1),
        window=w,
    )


@dataclass(frozen=True, slots=True)
class RingKVCache:
    """A fixed-capacity window for one-token decoding (``vesper/attention.py:63-82``): ``k, v
    [b, window, hkv, dk]`` (keys rotated), ``pos [b, window]`` int64, ``valid [b, window]`` bool.
    A token at position ``p`` lives in slot ``p % window``; slots are not in age order and
    visibility is ``valid`` with the window mask on positions. Its shapes never change, so a
    captured decode step carries it; this build's decode step updates it in place."""

    k: Tensor
    v: Tensor
    pos: Tensor
    valid: Tensor
    window: int


def kv_ring_empty(b: int, hkv: int, dk: int, window: int, dtype: torch.dtype, device: torch.device) -> RingKVCache:
    """Every slot unwritten: zero keys and values, positions 0, valid False (``vesper/attention.py:85-106``)."""
    if window < 1:
        msg = f"window must be at least 1, got {window}"
        raise ValueError(msg)
    return RingKVCache(
        k=torch.zeros(b, window, hkv, dk, dtype=dtype, device=device),
        v=torch.zeros(b, window, hkv, dk, dtype=dtype, device=device),
        pos=torch.zeros(b, window, dtype=torch.long, device=device),
        valid=torch.zeros(b, window, dtype=torch.bool, device=device),
        window=window,
    )


def ring_from_cache(cache: KVCache) -> RingKVCache:
    """The ring holding a chronological cache's entries, each in slot ``pos % window`` (the
    switch from a chunked prefill to one-token decoding)."""
    b, m, hkv, dk = cache.k.shape
    ring = kv_ring_empty(b, hkv, dk, cache.window, cache.k.dtype, cache.k.device)
    if m:
        slot = cache.pos % cache.window  # [b, m]
        at = slot[:, :, None, None].expand(b, m, hkv, dk)
        ring.k.scatter_(1, at, cache.k)
        ring.v.scatter_(1, at, cache.v)
        ring.pos.scatter_(1, slot, cache.pos)
        ring.valid.scatter_(1, slot, torch.ones_like(slot, dtype=torch.bool))
    return ring


class WindowedAttention(nn.Module):
    """Projections, rotary, windowed softmax over cache and chunk, output projection."""

    def __init__(self, d: int, heads: int, kv_groups: int, head_dim: int, window: int, rotary_base: float,
                 generator: torch.Generator | None = None) -> None:  # fmt: skip
        """The reference's initialization, draw for draw (``vesper/attention.py:226-267``)."""
        super().__init__()
        if heads % kv_groups != 0:
            msg = f"heads ({heads}) must be divisible by kv_groups ({kv_groups})"
            raise ValueError(msg)
        if window < 1:
            msg = f"window must be at least 1, got {window}"
            raise ValueError(msg)
        if not 1.0 < rotary_base < float("inf"):
            msg = f"rotary base must be finite and above 1, got {rotary_base}"
            raise ValueError(msg)
        self.heads, self.kv_heads, self.head_dim = heads, heads // kv_groups, head_dim
        self.window, self.rotary_base = window, rotary_base
        std = 1.0 / math.sqrt(d)
        kv = self.kv_heads * head_dim
        self.w_q = nn.Parameter(torch.randn(heads * head_dim, d, generator=generator) * std)
        self.w_k = nn.Parameter(torch.randn(kv, d, generator=generator) * std)
        self.w_v = nn.Parameter(torch.randn(kv, d, generator=generator) * std)
        self.w_o = nn.Parameter(torch.randn(d, heads * head_dim, generator=generator) * std)

    def project(self, x: Tensor, pos: Tensor) -> tuple[Tensor, Tensor, Tensor]:
        """Rotated ``q [b,n,h,dk]``, rotated ``k [b,n,hkv,dk]`` and ``v``."""
        dims: Dims = {}
        check_shape("x", x, ("b", "n", "d"), dims)
        check_shape("pos", pos, ("b", "n"), dims, dtype=torch.long)
        if pos.shape[1] > 1:
            require((pos[:, 1:] - pos[:, :-1] == 1).all(), "pos: positions must be consecutive within a chunk")
        b, n = x.shape[0], x.shape[1]
        q = F.linear(x, self.w_q).view(b, n, self.heads, self.head_dim)
        k = F.linear(x, self.w_k).view(b, n, self.kv_heads, self.head_dim)
        v = F.linear(x, self.w_v).view(b, n, self.kv_heads, self.head_dim)
        return rotary(q, pos, self.rotary_base), rotary(k, pos, self.rotary_base), v

    def output(self, o: Tensor) -> Tensor:
        """``[b, n, h, dk] -> [b, n, d]``."""
        return F.linear(o.flatten(2), self.w_o)

    def attend(self, q: Tensor, k: Tensor, v: Tensor, pos: Tensor, cache: KVCache,
               compaction: Compaction | None = None) -> tuple[Tensor, KVCache]:  # fmt: skip
        """Windowed softmax over the cache and the chunk; the new cache.

        ``compaction`` (the loop's active set, its ``qpos`` offset by the cache length): only the
        active queries are computed, the halted ones' outputs are zero (the loop discards them).
        """
        dims: Dims = {"hkv": self.kv_heads, "dk": self.head_dim, "h": self.heads}
        check_shape("q", q, ("b", "n", "h", "dk"), dims)
        keys, vals = self._keys_values(q.dtype, k, v, pos, cache, dims)
        if dims["n"] == 0:
            return q.new_zeros(dims["b"], 0, self.w_o.shape[0]), cache
        w = self.window
        if compaction is None:
            o = window_attention(q, keys, vals, w)
        else:
            (qc,) = gather_rows(compaction, [q])
            oc = window_attention_active(qc, compaction.qpos, compaction.counts, keys, vals, w)
            (o,) = expand_rows(compaction, [oc])
        return self.output(o), kv_cache_push(cache, k, v, pos)

    def attend_packed(self, qc: Tensor, k: Tensor, v: Tensor, pos: Tensor, cache: KVCache,
                      compaction: Compaction) -> tuple[Tensor, KVCache]:  # fmt: skip
        """``attend`` with the queries of the active tokens only, packed at the front of each batch
        row as ``compaction`` packs them (``qc [b, n, h, dk]``, padding rows ignored), returning
        their outputs packed the same way (zero padding) BEFORE the output projection, and the new
        cache. The loop's compacted passes project those rows themselves."""
        dims: Dims = {"hkv": self.kv_heads, "dk": self.head_dim, "h": self.heads}
        check_shape("qc", qc, ("b", "n", "h", "dk"), dims)
        keys, vals = self._keys_values(qc.dtype, k, v, pos, cache, dims)
        if dims["n"] == 0:
            return qc.new_zeros(qc.shape), cache
        oc = window_attention_active(qc, compaction.qpos, compaction.counts, keys, vals, self.window)
        return oc, kv_cache_push(cache, k, v, pos)

    def _keys_values(self, dtype: torch.dtype, k: Tensor, v: Tensor, pos: Tensor, cache: KVCache,
                     dims: Dims) -> tuple[Tensor, Tensor]:  # fmt: skip
        """The checks of the chunk and the cache, and every position's keys and values (cache
        rows, then the chunk's) in ``dtype``."""
        check_shape("k", k, ("b", "n", "hkv", "dk"), dims)
        check_shape("v", v, ("b", "n", "hkv", "dk"), dims)
        check_shape("pos", pos, ("b", "n"), dims, dtype=torch.long)
        check_shape("cache.k", cache.k, ("b", "m", "hkv", "dk"), dims)
        check_shape("cache.v", cache.v, ("b", "m", "hkv", "dk"), dims)
        check_shape("cache.pos", cache.pos, ("b", "m"), dims, dtype=torch.long)
        if cache.window != self.window:
            msg = f"cache window {cache.window} does not match the layer's {self.window}"
            raise ContractError(msg)
        if dims["n"] == 0:
            return k, v
        if k.device.type != "cuda":
            msg = f"the windowed attention runs on CUDA only, got {k.device}"
            raise ContractError(msg)
        if dtype not in WINDOW_KERNEL_DTYPES:
            msg = f"q: dtype must be one of {WINDOW_KERNEL_DTYPES}, got {dtype}"
            raise ContractError(msg)
        kpos = torch.cat([cache.pos, pos], dim=1)
        require((kpos[:, 1:] - kpos[:, :-1] == 1).all(), "attend: cache and chunk positions must be consecutive")
        keys = torch.cat([cache.k.to(dtype), k.to(dtype)], dim=1)
        vals = torch.cat([cache.v.to(dtype), v.to(dtype)], dim=1)
        return keys, vals

    def attend_ring(self, q: Tensor, k: Tensor, v: Tensor, pos: Tensor, ring: RingKVCache) -> tuple[Tensor, RingKVCache]:
        """One decoding token per row over its ring and itself (``vesper/attention.py:298-338``):
        ``q [b,1,h,dk]``, ``k, v [b,1,hkv,dk]``, ``pos [b,1]``. One kernel (``vb_ring_attend``)
        attends and then writes the token into its slot ``pos % window``: the ring is updated IN
        PLACE and returned (the decode step's carried buffers)."""
        dims: Dims = {"hkv": self.kv_heads, "dk": self.head_dim, "h": self.heads, "one": 1, "w": self.window}
        check_shape("q", q, ("b", "one", "h", "dk"), dims)
        check_shape("k", k, ("b", "one", "hkv", "dk"), dims)
        check_shape("v", v, ("b", "one", "hkv", "dk"), dims)
        check_shape("pos", pos, ("b", "one"), dims, dtype=torch.long)
        check_shape("ring.k", ring.k, ("b", "w", "hkv", "dk"), dims)
        check_shape("ring.v", ring.v, ("b", "w", "hkv", "dk"), dims)
        check_shape("ring.pos", ring.pos, ("b", "w"), dims, dtype=torch.long)
        check_shape("ring.valid", ring.valid, ("b", "w"), dims, dtype=torch.bool)
        if ring.window != self.window:
            msg = f"ring window {ring.window} does not match the layer's {self.window}"
            raise ContractError(msg)
        if q.device.type != "cuda":
            msg = f"the ring attention runs on CUDA only, got {q.device}"
            raise ContractError(msg)
        dt = ring.k.dtype
        if dt not in WINDOW_KERNEL_DTYPES or ring.v.dtype != dt:
            msg = f"ring: dtype must be one of {WINDOW_KERNEL_DTYPES}, got {dt}"
            raise ContractError(msg)
        b = dims["b"]
        qc, kc, vc = (t.to(dt).contiguous() for t in (q, k, v))
        o = torch.empty_like(qc)
        from vesper_b200 import _lib  # noqa: PLC0415

        ws = _lib.workspace(
            _lib.query("vb_ring_attend_workspace", b, self.window, self.heads, self.kv_heads, self.head_dim), q.device
        )
        _lib.call(
            "vb_ring_attend", qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), ring.k.data_ptr(), ring.v.data_ptr(),
            ring.pos.data_ptr(), ring.valid.data_ptr(), pos.contiguous().data_ptr(), o.data_ptr(), ws.data_ptr(), b,
            self.window, self.heads, self.kv_heads, self.head_dim, self.window, _lib.DTYPE_CODE[dt],
            _lib.stream(q.device),
        )  # fmt: skip
        return self.output(o.to(q.dtype)), ring

    def forward(self, x: Tensor, pos: Tensor, cache: KVCache) -> tuple[Tensor, KVCache]:
        """``project`` then ``attend``."""
        q, k, v = self.project(x, pos)
        return self.attend(q, k, v, pos, cache)
