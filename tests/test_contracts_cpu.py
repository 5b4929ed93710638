"""The boundary's refusals, checked on a CPU-only machine before any kernel is reached.

The messages follow the reference's (vesper tests/test_delta_scan_fused.py:125-151): "dtype",
"axis", "CUDA only"; a CPU tensor never silently takes another path.
"""

from __future__ import annotations

import pytest
import torch

from vesper_b200 import _lib
from vesper_b200.contracts import ContractError, check_shape
from vesper_b200.kernels.delta_scan import delta_scan_fused_fp32
from vesper_b200.kernels.keys import fused_keys
from vesper_b200.kernels.norm import fused_rms_norm


def test_check_shape_binds_and_refuses_like_the_reference() -> None:
    dims: dict[str, int] = {}
    check_shape("a", torch.zeros(2, 3), ("b", "n"), dims)
    assert dims == {"b": 2, "n": 3}
    with pytest.raises(ContractError, match="axis 1 'n' is 4"):
        check_shape("c", torch.zeros(2, 4), ("b", "n"), dims)
    with pytest.raises(ContractError, match="expected rank"):
        check_shape("c", torch.zeros(2), ("b", "n"), dims)
    with pytest.raises(ContractError, match="dtype"):
        check_shape("c", torch.zeros(2, 3), ("b", "n"), dims, torch.bfloat16)


def test_a_cpu_tensor_is_refused_by_every_fused_op() -> None:
    z = torch.zeros(1, 4, 1, 8)
    with pytest.raises(ContractError, match="CUDA only"):
        delta_scan_fused_fp32(z, z, z, torch.zeros(1, 4, 1), torch.zeros(1, 1, 8, 8))
    with pytest.raises(ContractError, match="CUDA only"):
        fused_keys(torch.zeros(1, 4, 8), torch.zeros(1, 3, 8), torch.zeros(4, 8), 1)
    with pytest.raises(ContractError, match="CUDA only"):
        fused_rms_norm(torch.zeros(2, 8), torch.ones(8), 1e-3, 1e-6)


def test_shape_and_dtype_errors_come_before_the_device_check() -> None:
    q = torch.zeros(1, 8, 2, 16)
    with pytest.raises(ContractError, match="dtype"):
        delta_scan_fused_fp32(q.bfloat16(), q, q, torch.zeros(1, 8, 2), torch.zeros(1, 2, 16, 16))
    with pytest.raises(ContractError, match="axis"):
        delta_scan_fused_fp32(q, q[:, :4], q, torch.zeros(1, 8, 2), torch.zeros(1, 2, 16, 16))


def test_the_key_filter_refuses_statistics_off_an_8_byte_boundary() -> None:
    """Both key-filter entry points check the statistics buffer on the host before any launch
    (the addresses below are never dereferenced)."""
    bf16 = _lib.DTYPE_CODE[torch.bfloat16]
    aligned, odd = 1 << 20, (1 << 20) + 4
    with pytest.raises(_lib.KernelError, match="8-byte boundary"):
        _lib.call("vb_keys_fwd", aligned, aligned, aligned, aligned, odd, 1, 64, 128, 2, 4, 1e-6, bf16, None)
    with pytest.raises(_lib.KernelError, match="8-byte boundary"):
        _lib.call(
            "vb_keys_bwd", aligned, aligned, aligned, aligned, odd, aligned, aligned, None, aligned,
            1, 64, 128, 2, 4, 1e-6, bf16, None,
        )  # fmt: skip
