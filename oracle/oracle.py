"""TEST INFRASTRUCTURE ONLY: ctypes bindings of the float64 CPU oracle (``vesper_oracle.c``).

The oracle restates the reference's pure-PyTorch path (mstampfli/vesper-preview,
``vesper/recurrence.py``, ``vesper/column.py``, ``vesper/attention.py``) in plain C. Only the
tests, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs import this module, as the
checker or as the timed CPU port; the ``vesper_b200`` package never does.

Every function takes numpy arrays (any float dtype; converted to contiguous float64) and returns
float64 arrays in the reference's layouts.
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"

_lib: ctypes.CDLL | None = None
_P = ctypes.POINTER(ctypes.c_double)


def build() -> Path:
    """Compile the oracle with its Makefile (gcc, OpenMP); returns the library path."""
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        i, d, p, i64 = ctypes.c_int, ctypes.c_double, _P, ctypes.c_int64
        _lib.vo_delta_scan_fwd.argtypes = [i, i, i, i, p, p, p, p, p, p, p]
        _lib.vo_delta_scan_bwd.argtypes = [i, i, i, i, p, p, p, p, p, p, p, p, p, p, p, p]
        _lib.vo_keys_fwd.argtypes = [i, i, i, i, i, p, p, p, d, p]
        _lib.vo_keys_bwd.argtypes = [i, i, i, i, i, p, p, p, d, p, p, p, p]
        _lib.vo_rms_fwd.argtypes = [i64, i, p, p, d, d, p, p]
        _lib.vo_rms_bwd.argtypes = [i64, i, p, p, d, d, p, p, p]
        _lib.vo_window_attn_fwd.argtypes = [i, i, i, i, i, i, i, p, p, p, p, p]
        _lib.vo_window_attn_bwd.argtypes = [i, i, i, i, i, i, i, p, p, p, p, p, p, p]
        _lib.vo_num_threads.restype = ctypes.c_int
        _lib.vo_set_threads.argtypes = [i]
        _lib.vo_set_threads.restype = ctypes.c_int
    return _lib


def _f64(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float64))


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(_P)


def threads() -> int:
    """OpenMP threads the oracle uses (``OMP_NUM_THREADS`` or all cores)."""
    return int(lib().vo_num_threads())


def set_threads(n: int) -> int:
    """Use ``n`` OpenMP threads from now on (overriding ``OMP_NUM_THREADS``); returns the count."""
    return int(lib().vo_set_threads(int(n)))


def usable_cores() -> int:
    """The CPUs this process may run on (its affinity mask), whatever ``OMP_NUM_THREADS`` says."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


KEY_NORM_FLOOR = 1e-6  # recurrence.py:27
RMS_EPS = 1e-6  # column.py:55
RMS_FLOOR = 1e-3  # column.py:56


def delta_scan(q, k, v, beta, s0):
    """``(o [B,T,H,D], s_n [B,H,D,D])`` of the delta rule, token by token, in float64."""
    q, k, v, beta, s0 = map(_f64, (q, k, v, beta, s0))
    B, T, H, D = q.shape
    o = np.zeros_like(q)
    sn = np.zeros_like(s0)
    lib().vo_delta_scan_fwd(B, T, H, D, *map(_ptr, (q, k, v, beta, s0, o, sn)))
    return o, sn


def delta_scan_grads(q, k, v, beta, s0, dout, dsn):
    """Gradients ``(dq, dk, dv, dbeta, ds0)`` of ``sum(o*dout) + sum(s_n*dsn)``."""
    q, k, v, beta, s0, dout, dsn = map(_f64, (q, k, v, beta, s0, dout, dsn))
    B, T, H, D = q.shape
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    dbeta, ds0 = np.zeros_like(beta), np.zeros_like(s0)
    lib().vo_delta_scan_bwd(
        B, T, H, D, *map(_ptr, (q, k, v, beta, s0, dout, dsn, dq, dk, dv, dbeta, ds0))
    )
    return dq, dk, dv, dbeta, ds0


def keys(z, hist, taps, heads, floor=KEY_NORM_FLOOR):
    """Normalized filtered keys ``[B,T,heads,W/heads]`` (column.py:255-289)."""
    z, hist, taps = map(_f64, (z, hist, taps))
    B, T, W = z.shape
    K = taps.shape[0]
    out = np.zeros((B, T, W))
    lib().vo_keys_fwd(B, T, W, heads, K, _ptr(z), _ptr(hist), _ptr(taps), floor, _ptr(out))
    return out.reshape(B, T, heads, W // heads)


def keys_grads(z, hist, taps, heads, gk, floor=KEY_NORM_FLOOR):
    """``(dz [B,T,W], dhist [B,K-1,W], dtaps [K,W])`` of ``sum(keys * gk)``."""
    z, hist, taps, gk = map(_f64, (z, hist, taps, gk))
    B, T, W = z.shape
    K = taps.shape[0]
    dz, dhist, dtaps = np.zeros((B, T, W)), np.zeros((B, K - 1, W)), np.zeros((K, W))
    lib().vo_keys_bwd(
        B, T, W, heads, K, _ptr(z), _ptr(hist), _ptr(taps), floor, _ptr(gk.reshape(B, T, W)),
        _ptr(dz), _ptr(dhist), _ptr(dtaps),
    )  # fmt: skip
    return dz, dhist, dtaps


def next_history(z, hist):
    """The newest ``K-1`` rows of ``cat(hist, z)`` (column.py:281-282, :288)."""
    z, hist = _f64(z), _f64(hist)
    full = np.concatenate([hist, z], axis=1)
    return full[:, z.shape[1] :].copy()


def rms_norm(x, g, floor=RMS_FLOOR, eps=RMS_EPS):
    """``(y, inv)`` of the scale-safe RMSNorm over the last axis (column.py:159-188)."""
    x, g = _f64(x), _f64(g)
    W = x.shape[-1]
    rows = x.size // W if W else 0
    y = np.zeros_like(x)
    inv = np.zeros(rows)
    lib().vo_rms_fwd(rows, W, _ptr(x), _ptr(g), floor, eps, _ptr(y), _ptr(inv))
    return y, inv.reshape(x.shape[:-1])


def rms_norm_grads(x, g, dy, floor=RMS_FLOOR, eps=RMS_EPS):
    """``(dx, dg)`` of ``sum(rms_norm(x, g) * dy)``."""
    x, g, dy = _f64(x), _f64(g), _f64(dy)
    W = x.shape[-1]
    rows = x.size // W if W else 0
    dx, dg = np.zeros_like(x), np.zeros(W)
    lib().vo_rms_bwd(rows, W, _ptr(x), _ptr(g), floor, eps, _ptr(dy), _ptr(dx), _ptr(dg))
    return dx, dg


def window_attention(q, keys_, values, window):
    """``o [B,n,H,D]`` of q over ``keys, values [B, m+n, Hkv, D]`` (cache first)."""
    q, keys_, values = map(_f64, (q, keys_, values))
    B, n, H, D = q.shape
    L, Hkv = keys_.shape[1], keys_.shape[2]
    o = np.zeros_like(q)
    lib().vo_window_attn_fwd(
        B, n, L, H, Hkv, D, window, _ptr(q), _ptr(keys_), _ptr(values), _ptr(o), None
    )
    return o


def window_attention_grads(q, keys_, values, window, dout):
    """``(dq, dkeys, dvalues)`` of ``sum(o * dout)``."""
    q, keys_, values, dout = map(_f64, (q, keys_, values, dout))
    B, n, H, D = q.shape
    L, Hkv = keys_.shape[1], keys_.shape[2]
    dq, dk, dv = np.zeros_like(q), np.zeros_like(keys_), np.zeros_like(values)
    lib().vo_window_attn_bwd(
        B, n, L, H, Hkv, D, window, *map(_ptr, (q, keys_, values, dout, dq, dk, dv))
    )
    return dq, dk, dv


def available() -> bool:
    try:
        lib()
    except OSError:
        return False
    return True


if __name__ == "__main__":  # pragma: no cover
    print(build(), threads(), os.cpu_count())
