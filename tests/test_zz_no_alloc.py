"""The allocation-free RMSNorm backward, ``vb_rms_norm_bwd_noalloc``, through the C ABI.

Some callers cannot allocate device memory at the moment they need the gradient: a plugin host
that hands the library a fixed memory budget, a loop that must never allocate, a capture or a
memory plan that an allocation would break. For them the library keeps the gain gradient's
partial sums in a fixed 4 MiB device array instead of a caller-provided workspace. This test
checks, on a GPU, that two calls in a row (of different sizes, so that the second finds the first
one's partial sums in the shared array) give the same dx and gain gradient as the workspace entry
point ``vb_rms_norm_bwd``, within the tolerance the norm tests use, and that a call larger than
the array is refused with the limit in the message.

The file is named to be collected last, so that a run stopping at the first failure has already
run every other test.
"""

from __future__ import annotations

import pytest
import torch

from vesper_b200 import _lib

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")
TOL = 2e-5


def _forward(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    inv = torch.empty(x.shape[0], dtype=torch.float32, device=CUDA)
    y = torch.empty_like(x)
    _lib.call("vb_rms_norm_fwd", x.data_ptr(), w.data_ptr(), y.data_ptr(), inv.data_ptr(), x.shape[0],
              x.shape[1], 1e-3, 1e-6, _lib.DTYPE_CODE[x.dtype], _lib.stream(CUDA))
    return inv


def _with_workspace(x, w, dy, inv):
    dx = torch.empty_like(x)
    dg = torch.empty(x.shape[1], dtype=torch.float32, device=CUDA)
    ws = _lib.workspace(_lib.query("vb_rms_norm_bwd_workspace", x.shape[0], x.shape[1]), CUDA)
    _lib.call("vb_rms_norm_bwd", x.data_ptr(), w.data_ptr(), dy.data_ptr(), inv.data_ptr(), dx.data_ptr(),
              dg.data_ptr(), ws.data_ptr(), x.shape[0], x.shape[1], _lib.DTYPE_CODE[x.dtype], _lib.stream(CUDA))
    return dx, dg


def _without_allocation(x, w, dy, inv):
    dx = torch.empty_like(x)
    dg = torch.empty(x.shape[1], dtype=torch.float32, device=CUDA)
    _lib.call("vb_rms_norm_bwd_noalloc", x.data_ptr(), w.data_ptr(), dy.data_ptr(), inv.data_ptr(),
              dx.data_ptr(), dg.data_ptr(), x.shape[0], x.shape[1], _lib.DTYPE_CODE[x.dtype], _lib.stream(CUDA))
    return dx, dg


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_two_calls_in_a_row_match_the_workspace_entry_point(dtype: torch.dtype) -> None:
    g = torch.Generator(device=CUDA).manual_seed(3)
    for rows, width in ((4096, 1024), (300, 512)):  # the second call is smaller than the first
        x = (3 * torch.randn(rows, width, device=CUDA, generator=g)).to(dtype)
        w = 1 + 0.1 * torch.randn(width, device=CUDA, generator=g)
        dy = torch.randn(rows, width, device=CUDA, generator=g).to(dtype)
        inv = _forward(x, w)
        want_dx, want_dg = _with_workspace(x, w, dy, inv)
        got_dx, got_dg = _without_allocation(x, w, dy, inv)
        torch.cuda.synchronize()
        torch.testing.assert_close(got_dx.float(), want_dx.float(), rtol=TOL, atol=TOL)
        torch.testing.assert_close(got_dg, want_dg, rtol=TOL, atol=TOL)


def test_a_call_one_row_beyond_the_fixed_scratch_is_refused() -> None:
    # at width 1024 the array holds the partial sums of 65536 rows (1024 blocks of 64 rows); one
    # row more needs a 1025th block of partial sums: refused before any pointer is touched
    rows, width = 65536 + 1, 1024
    with pytest.raises(_lib.KernelError, match="fixed scratch"):
        _lib.call("vb_rms_norm_bwd_noalloc", None, None, None, None, None, None, rows, width,
                  _lib.DTYPE_CODE[torch.float32], _lib.stream(CUDA))


def test_a_call_that_fills_the_fixed_scratch_exactly_is_accepted_and_matches() -> None:
    # 65536 rows at width 1024: every one of the array's 2^20 partial sums is written and read
    g = torch.Generator(device=CUDA).manual_seed(4)
    rows, width = 65536, 1024
    x = torch.randn(rows, width, device=CUDA, generator=g).to(torch.bfloat16)
    w = 1 + 0.1 * torch.randn(width, device=CUDA, generator=g)
    dy = torch.randn(rows, width, device=CUDA, generator=g).to(torch.bfloat16)
    inv = _forward(x, w)
    want_dx, want_dg = _with_workspace(x, w, dy, inv)
    got_dx, got_dg = _without_allocation(x, w, dy, inv)
    torch.cuda.synchronize()
    torch.testing.assert_close(got_dx.float(), want_dx.float(), rtol=TOL, atol=TOL)
    torch.testing.assert_close(got_dg, want_dg, rtol=TOL, atol=TOL)
