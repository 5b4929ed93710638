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


def require(condition: torch.Tensor, message: str) -> None:
    """A value contract computed on the device (``vesper/contracts.py:104-131``'s ``require``).

    Eagerly the one-element bool is read back and a false one raises ``ContractError(message)``.
    While a CUDA graph is being captured a read-back would end the capture, so the violation is
    recorded instead: bit 4 is ORed into the device status word (``_lib.status_word``), which
    ``_lib.check_status`` reads after the replay and raises on. Unlike the reference, no device
    assert is ever recorded: a violated contract never faults the GPU.
    """
    if condition.dtype != torch.bool or condition.numel() != 1:
        msg = f"require: the condition must be one bool, got {condition.dtype} {tuple(condition.shape)}"
        raise ContractError(msg)
    if condition.is_cuda and torch.cuda.is_current_stream_capturing():
        from vesper_b200 import _lib  # noqa: PLC0415  # the library loads only for device work

        word = _lib.status_word(condition.device)
        word.bitwise_or_(condition.logical_not().reshape(1).to(torch.int32) * 4)
        return
    if not bool(condition.item()):
        raise ContractError(message)


def check_ids(name: str, tensor: torch.Tensor, spec: DimSpec, dims: Dims, vocab: int) -> torch.Tensor:
    """Ids of ``int32`` or ``int64`` within ``[0, vocab)``, returned as ``int64``
    (``vesper/contracts.py:75-101``)."""
    check_shape(name, tensor, spec, dims)
    if tensor.dtype not in (torch.int32, torch.int64):
        msg = f"{name}: dtype must be int32 or int64, got {tensor.dtype}"
        raise ContractError(msg)
    if tensor.numel() > 0:
        require(((tensor >= 0) & (tensor < vocab)).all(), f"{name}: every id must lie in [0, vocab={vocab})")
    return tensor.long()
