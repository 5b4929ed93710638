"""Tensor contracts at the kernel boundary: the reference's ``check_shape`` and ``ContractError``.

Mirrors ``vesper/contracts.py:31-71`` of mstampfli/vesper-preview (same error type, same message
fragments: "expected rank", "axis", "dtype must be"), so callers and tests that match the
reference's messages keep working against these kernels.
"""

from __future__ import annotations

import torch

Dims = dict[str, int]
DimSpec = tuple[str | int, ...]


class ContractError(ValueError):
    """A tensor did not meet its contract (rank, dimension binding, dtype or device)."""


def check_shape(
    name: str,
    tensor: torch.Tensor,
    spec: DimSpec,
    dims: Dims,
    dtype: torch.dtype | None = None,
) -> None:
    """Check ``tensor`` against ``spec`` and bind unbound dimension names in ``dims``."""
    shape = tuple(tensor.shape)
    if len(shape) != len(spec):
        msg = f"{name}: expected rank {len(spec)} {spec}, got shape {shape}"
        raise ContractError(msg)
    for axis, (want, got) in enumerate(zip(spec, shape, strict=True)):
        if isinstance(want, int):
            if got != want:
                msg = f"{name}: axis {axis} must be {want}, got {got} (shape {shape})"
                raise ContractError(msg)
            continue
        bound = dims.get(want)
        if bound is None:
            dims[want] = got
        elif bound != got:
            msg = f"{name}: axis {axis} '{want}' is {got}, but '{want}' = {bound} elsewhere"
            raise ContractError(msg)
    if dtype is not None and tensor.dtype != dtype:
        msg = f"{name}: dtype must be {dtype}, got {tensor.dtype}"
        raise ContractError(msg)


def require_cuda(what: str, first: torch.Tensor, **others: torch.Tensor | None) -> None:
    """All tensors on one CUDA device; the messages of kernels/delta_scan.py:109-117."""
    if first.device.type != "cuda":
        msg = f"the {what} runs on CUDA only, got {first.device}"
        raise ContractError(msg)
    for name, tensor in others.items():
        if tensor is not None and tensor.device != first.device:
            msg = f"{name} is on {tensor.device}, the first input on {first.device}"
            raise ContractError(msg)
