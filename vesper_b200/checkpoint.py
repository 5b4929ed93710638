"""Checkpoints of the training step: weights, optimizer and the carried per-pass states.

The format of the reference's trainer checkpoint (``vesper/train.py:907-951`` ``_state_record`` /
``_states_from_record``, ``:993-1053`` ``checkpoint``, ``:1068-1130`` ``restore``): a directory of
``model.pt`` (the model's ``state_dict``), ``optimizer.pt`` (AdamW's), ``states.pt`` and
``train.json``, with ``manifest.json`` holding each file's SHA-256. ``states.pt`` is
``{"groups": [{"states": record, "stream": None}, ...], "mixer": None}``; a record is, per column,
``{"h": [t_max float32 [b,h,dk,dk]], "kv": [{"k", "v", "pos", "window"}] * t_max,
"key_history": [t_max [b,K-1,d]]}`` (plain containers, ``weights_only`` loads). A data-parallel
run stores one group per rank (its own batch rows: the reference's independent streams), so a
resumed rank continues exactly its own rows. The data stream's packing state and the mixer are
outside this build's path and are stored as ``None``.

The directory is written beside its destination and published by one rename, so a failed save
leaves nothing behind; an existing checkpoint is never overwritten (the reference's rule).
``restore`` verifies every hash, loads on the CPU, validates each state against the model's
geometry (``check_column_state``, the reference's ``vesper/column.py:606-678`` rules and messages)
and copies everything IN PLACE into the trainer's existing tensors, so a captured step graph
stays valid across a restore.
"""

from __future__ import annotations

import hashlib
import io
import json
import os
import shutil
import tempfile
from collections.abc import Sequence
from pathlib import Path
from typing import TYPE_CHECKING

import torch
import torch.distributed as dist
from torch import Tensor

from vesper_b200.attention import KVCache
from vesper_b200.column import ColumnShape, ColumnState, state_tensors, with_state_tensors
from vesper_b200.contracts import Dims, check_shape

if TYPE_CHECKING:
    from vesper_b200.train import TrainStep

FILES = ("model.pt", "optimizer.pt", "states.pt", "train.json")
SCHEMA = 1


def check_column_state(state: ColumnState, shape: ColumnShape, t_max: int) -> None:
    """Refuse a carried state this geometry and pass count cannot run (``vesper/column.py:606-678``).

    Raises:
        ValueError: on a pass count other than ``t_max``, a window other than the shape's, a
            recurrent state or key history that is not real float32 or wider, an attention window
            that is not real floating point, or a tensor on another device than ``h[0]``.
        ContractError: on a tensor shape that does not match the geometry, or batch sizes that
            differ between fields.
    """
    counts = {len(state.h), len(state.kv), len(state.key_history)}
    if counts != {t_max}:
        msg = f"state has {sorted(counts)} passes in its fields, the loop runs {t_max}"
        raise ValueError(msg)
    dims: Dims = {"h": shape.heads, "hkv": shape.kv_heads, "dk": shape.head_dim, "d": shape.d, "w": shape.key_history}
    device = state.h[0].device
    for t in range(t_max):
        h, cache, history = state.h[t], state.kv[t], state.key_history[t]
        check_shape(f"h[{t}]", h, ("b", "h", "dk", "dk"), dims)
        check_shape(f"key_history[{t}]", history, ("b", "w", "d"), dims)
        check_shape(f"kv[{t}].k", cache.k, ("b", f"m{t}", "hkv", "dk"), dims)
        check_shape(f"kv[{t}].v", cache.v, ("b", f"m{t}", "hkv", "dk"), dims)
        check_shape(f"kv[{t}].pos", cache.pos, ("b", f"m{t}"), dims, dtype=torch.long)
        if cache.window != shape.window:
            msg = f"kv[{t}] has window {cache.window}, the column has {shape.window}"
            raise ValueError(msg)
        for name, tensor in ((f"h[{t}]", h), (f"key_history[{t}]", history)):
            if not tensor.dtype.is_floating_point or torch.promote_types(tensor.dtype, torch.float32) != tensor.dtype:
                msg = f"{name} is {tensor.dtype}; carried states are real float32 or wider"
                raise ValueError(msg)
        for name, tensor in ((f"kv[{t}].k", cache.k), (f"kv[{t}].v", cache.v)):
            if not tensor.dtype.is_floating_point:
                msg = f"{name} is {tensor.dtype}; attention windows are real floating point"
                raise ValueError(msg)
        for name, tensor in ((f"h[{t}]", h), (f"key_history[{t}]", history), (f"kv[{t}].k", cache.k),
                             (f"kv[{t}].v", cache.v), (f"kv[{t}].pos", cache.pos)):  # fmt: skip
            if tensor.device != device:
                msg = f"{name} is on {tensor.device}, h[0] on {device}; one device"
                raise ValueError(msg)


def state_record(states: Sequence[ColumnState]) -> list[dict[str, object]]:
    """The carried states as plain containers (``vesper/train.py:907-924``), detached, on the CPU."""
    cpu = [torch.Tensor.detach(t).cpu() for t in state_tensors(states)]
    plain = with_state_tensors(states, cpu)
    return [
        {
            "h": list(s.h),
            "kv": [{"k": c.k, "v": c.v, "pos": c.pos, "window": c.window} for c in s.kv],
            "key_history": list(s.key_history),
        }
        for s in plain
    ]


def states_from_record(record: list[dict[str, object]], shape: ColumnShape, t_max: int) -> list[ColumnState]:
    """The inverse of ``state_record``, each column's state validated (``vesper/train.py:927-951``)."""
    out: list[ColumnState] = []
    for column in record:
        caches = column["kv"]
        state = ColumnState(
            h=tuple(column["h"]),  # type: ignore[arg-type]
            kv=tuple(KVCache(k=c["k"], v=c["v"], pos=c["pos"], window=int(c["window"])) for c in caches),  # type: ignore[union-attr, index]
            key_history=tuple(column["key_history"]),  # type: ignore[arg-type]
        )
        check_column_state(state, shape, t_max)
        out.append(state)
    return out


def _sha256(data: bytes) -> str:
    return hashlib.sha256(data).hexdigest()


def _torch_bytes(obj: object) -> bytes:
    buf = io.BytesIO()
    torch.save(obj, buf)
    return buf.getvalue()


def _gather_records(record: list[dict[str, object]], distributed: bool) -> list[list[dict[str, object]]]:
    """Every rank's record on rank 0 (in rank order); the single record without a process group."""
    if not distributed:
        return [record]
    everyone: list[object] = [None] * dist.get_world_size()
    dist.all_gather_object(everyone, record)
    return everyone  # type: ignore[return-value]


def save(path: str | os.PathLike[str], trainer: TrainStep, *, reason: str = "interval") -> Path | None:
    """Write the trainer's checkpoint directory at ``path``; returns the manifest's path on the
    writing rank (rank 0), None on the others. Every rank must call it (the carried states of all
    ranks are gathered to rank 0, one group per rank).

    Raises:
        ValueError: when ``path`` already holds a checkpoint.
    """
    path = Path(path)
    distributed = trainer.distributed and dist.is_initialized()
    rank = dist.get_rank() if distributed else 0
    states = with_state_tensors(trainer.templates, trainer.state)
    records = _gather_records(state_record(states), distributed)
    if rank != 0:
        return None
    if path.exists():
        msg = f"{path}: a checkpoint already exists there"
        raise ValueError(msg)
    blobs = {
        "model.pt": _torch_bytes({k: v.detach().cpu() for k, v in trainer.model.state_dict().items()}),
        "optimizer.pt": _torch_bytes(_cpu(trainer.opt.state_dict())),
        "states.pt": _torch_bytes({"groups": [{"states": r, "stream": None} for r in records], "mixer": None}),
        "train.json": json.dumps({
            "schema": SCHEMA, "reason": reason,
            "progress": {"step": trainer.steps, "position": int(trainer.pos[0, 0].item())},
            "layout": {"groups": len(records), "rows_per_group": trainer.b, "tokens_per_row": trainer.n},
        }, sort_keys=True).encode(),  # fmt: skip
    }
    path.parent.mkdir(parents=True, exist_ok=True)
    staging = Path(tempfile.mkdtemp(prefix=f".{path.name}.", suffix=".staging", dir=path.parent))
    try:
        partial = staging / path.name
        partial.mkdir()
        for name, data in blobs.items():
            (partial / name).write_bytes(data)
        manifest = {name: _sha256(data) for name, data in blobs.items()}
        (partial / "manifest.json").write_text(json.dumps(manifest, sort_keys=True))
        os.rename(partial, path)
    finally:
        shutil.rmtree(staging, ignore_errors=True)
    return path / "manifest.json"


def _cpu(obj: object) -> object:
    if isinstance(obj, Tensor):
        return obj.detach().cpu()
    if isinstance(obj, dict):
        return {k: _cpu(v) for k, v in obj.items()}
    if isinstance(obj, list | tuple):
        return type(obj)(_cpu(v) for v in obj)
    return obj


def _verified(path: Path) -> dict[str, bytes]:
    try:
        manifest = json.loads((path / "manifest.json").read_text())
    except (OSError, ValueError) as exc:
        msg = f"{path}: no readable manifest ({exc})"
        raise ValueError(msg) from exc
    blobs = {}
    for name in FILES:
        try:
            data = (path / name).read_bytes()
        except OSError as exc:
            msg = f"{path / name}: missing"
            raise ValueError(msg) from exc
        if manifest.get(name) != _sha256(data):
            msg = f"{path / name}: its SHA-256 does not match the manifest"
            raise ValueError(msg)
        blobs[name] = data
    return blobs


def _copy_into(dst: object, src: object, where: str) -> None:
    """Copy ``src`` into the existing tensors of ``dst`` (same structure), in place."""
    if isinstance(dst, Tensor):
        if not isinstance(src, Tensor) or src.shape != dst.shape:
            msg = f"{where}: shape {getattr(src, 'shape', None)} does not fit {tuple(dst.shape)}"
            raise ValueError(msg)
        with torch.no_grad():
            dst.copy_(src.to(dst.dtype))
        return
    if isinstance(dst, dict):
        for k, v in dst.items():
            if k not in src:  # type: ignore[operator]
                msg = f"{where}: {k!r} missing"
                raise ValueError(msg)
            _copy_into(v, src[k], f"{where}.{k}")  # type: ignore[index]
        return
    if isinstance(dst, list | tuple):
        for i, (a, b) in enumerate(zip(dst, src, strict=True)):  # type: ignore[call-overload]
            _copy_into(a, b, f"{where}[{i}]")


def restore(path: str | os.PathLike[str], trainer: TrainStep) -> dict[str, object]:
    """Load a checkpoint written by ``save`` into ``trainer`` in place; returns ``train.json``.

    A data-parallel rank takes group ``rank`` (its own rows); the layout must match this run.

    Raises:
        ValueError: on a missing or changed file, another layout, or a state this model cannot run.
    """
    path = Path(path)
    blobs = _verified(path)
    record = json.loads(blobs["train.json"])
    distributed = trainer.distributed and dist.is_initialized()
    rank, world = (dist.get_rank(), dist.get_world_size()) if distributed else (0, 1)
    layout = record["layout"]
    if layout != {"groups": world, "rows_per_group": trainer.b, "tokens_per_row": trainer.n}:
        msg = f"{path}: checkpoint of layout {layout}; this run has {world} groups of {trainer.b} x {trainer.n}"
        raise ValueError(msg)
    model_sd = torch.load(io.BytesIO(blobs["model.pt"]), weights_only=True, map_location="cpu")
    opt_sd = torch.load(io.BytesIO(blobs["optimizer.pt"]), weights_only=True, map_location="cpu")
    saved = torch.load(io.BytesIO(blobs["states.pt"]), weights_only=True, map_location="cpu")
    states = states_from_record(saved["groups"][rank]["states"], trainer.model.shape, trainer.model.t_max)
    for name, p in trainer.model.state_dict().items():
        _copy_into(p, model_sd[name], f"model.{name}")
    current = trainer.opt.state_dict()
    if not current["state"]:
        # an optimizer that has not stepped yet: load the state whole (no graph holds it yet)
        trainer.opt.load_state_dict(opt_sd)
    else:
        _copy_into(current["state"], {int(k): v for k, v in opt_sd["state"].items()}, "optimizer.state")
        for cur_group, saved_group in zip(trainer.opt.param_groups, opt_sd["param_groups"], strict=True):
            for key, value in saved_group.items():
                if key == "params":
                    continue
                if isinstance(cur_group[key], Tensor):
                    _copy_into(cur_group[key], value, f"optimizer.{key}")
                else:
                    cur_group[key] = value
    flat = state_tensors(states)
    shapes_match = len(flat) == len(trainer.state) and all(
        a.shape == b.shape for a, b in zip(flat, trainer.state, strict=False))  # fmt: skip
    if shapes_match:
        for i, (dst, src) in enumerate(zip(trainer.state, flat, strict=True)):
            _copy_into(dst, src, f"states[{i}]")
    elif trainer.graph is None:
        # a trainer that has not run its first chunk yet holds cold (empty-window) states:
        # it takes the checkpoint's steady-state ones as its templates
        trainer.adopt_states(states)
    else:
        msg = f"{path}: the checkpoint's carried states do not fit the captured step's"
        raise ValueError(msg)
    position = int(record["progress"]["position"])
    with torch.no_grad():
        trainer.pos.copy_(torch.arange(trainer.n, device=trainer.pos.device).add(position).expand_as(trainer.pos))
    return record
