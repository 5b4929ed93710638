"""The training checkpoint's format on the CPU: the carried-state record, its validation, and a
two-rank (``gloo``) save and restore in which each rank gets back exactly its own rows.

``vesper_b200.checkpoint`` writes the reference trainer's layout (``vesper/train.py:907-1130``):
``model.pt``, ``optimizer.pt``, ``states.pt`` (one group of carried per-pass states per stream,
here per data-parallel rank), ``train.json`` and a SHA-256 manifest. The trainer here is a CPU
stand-in with the attributes the module reads (the real one needs a GPU; the GPU test resumes a
real ``TrainStep``).
"""

from __future__ import annotations

import json
import os
import socket
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vesper_b200 import checkpoint
from vesper_b200.attention import KVCache
from vesper_b200.column import ColumnShape, ColumnState, init_column_state, state_tensors
from vesper_b200.contracts import ContractError
from vesper_b200.model import Vesper

SHAPE = ColumnShape(d=32, heads=2, kv_groups=2, head_dim=16, window=8, rotary_base=10000.0, ffn_mult=2, block=16,
                    key_conv=4)  # fmt: skip
COLUMNS, T_MAX, B, N = 2, 3, 2, 16


def _filled_states(seed: int) -> list[ColumnState]:
    """Steady-state carried states (full windows) with seeded values."""
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(COLUMNS):
        cold = init_column_state(SHAPE, B, T_MAX, torch.float32, torch.device("cpu"))
        kv = tuple(KVCache(torch.randn(B, SHAPE.window, SHAPE.kv_heads, SHAPE.head_dim, generator=g).bfloat16(),
                           torch.randn(B, SHAPE.window, SHAPE.kv_heads, SHAPE.head_dim, generator=g).bfloat16(),
                           torch.arange(SHAPE.window).expand(B, SHAPE.window).contiguous() + 40, SHAPE.window)
                   for _ in range(T_MAX))  # fmt: skip
        out.append(ColumnState(h=tuple(torch.randn_like(h) for h in cold.h), kv=kv,
                               key_history=tuple(torch.randn_like(z) for z in cold.key_history)))  # fmt: skip
    return out


def _trainer(seed: int, distributed: bool = False) -> SimpleNamespace:
    model = Vesper(SHAPE, 64, COLUMNS, T_MAX, 0.01, torch.Generator().manual_seed(seed))
    opt = torch.optim.AdamW(model.parameters(), lr=1e-3)
    for p in model.parameters():  # one optimizer step so that its state exists
        p.grad = torch.ones_like(p) * 1e-3
    opt.step()
    templates = _filled_states(seed)
    trainer = SimpleNamespace(model=model, opt=opt, templates=templates, state=state_tensors(templates), steps=5,
                              pos=torch.arange(N).expand(B, N).contiguous() + 5 * N, b=B, n=N, graph=None,
                              distributed=distributed)  # fmt: skip
    return trainer


def test_the_state_record_round_trips_and_is_validated() -> None:
    states = _filled_states(1)
    record = checkpoint.state_record(states)
    assert set(record[0]) == {"h", "kv", "key_history"} and len(record) == COLUMNS
    back = checkpoint.states_from_record(record, SHAPE, T_MAX)
    for a, b in zip(state_tensors(states), state_tensors(back), strict=True):
        assert torch.equal(a, b)
    with pytest.raises(ValueError, match="passes"):
        checkpoint.states_from_record(record, SHAPE, T_MAX + 1)
    bad = checkpoint.state_record(states)
    bad[0]["h"][1] = bad[0]["h"][1].bfloat16()
    with pytest.raises(ValueError, match="float32 or wider"):
        checkpoint.states_from_record(bad, SHAPE, T_MAX)
    bad = checkpoint.state_record(states)
    bad[1]["kv"][0]["window"] = SHAPE.window + 1
    with pytest.raises(ValueError, match="window"):
        checkpoint.states_from_record(bad, SHAPE, T_MAX)
    bad = checkpoint.state_record(states)
    bad[0]["key_history"][2] = bad[0]["key_history"][2][:, :1]
    with pytest.raises(ContractError, match="axis"):
        checkpoint.states_from_record(bad, SHAPE, T_MAX)


def test_save_then_restore_into_another_trainer_is_exact(tmp_path: Path) -> None:
    a, b = _trainer(1), _trainer(2)
    manifest = checkpoint.save(tmp_path / "ckpt", a)
    assert manifest is not None and manifest.exists()
    files = json.loads(manifest.read_text())
    assert set(files) == set(checkpoint.FILES)
    record = checkpoint.restore(tmp_path / "ckpt", b)
    assert record["progress"]["step"] == 5
    for (na, pa), (nb, pb) in zip(a.model.state_dict().items(), b.model.state_dict().items(), strict=True):
        assert na == nb and torch.equal(pa, pb), na
    for x, y in zip(a.state, b.state, strict=True):
        assert torch.equal(x, y)
    sa, sb = a.opt.state_dict()["state"], b.opt.state_dict()["state"]
    for k in sa:
        for key in sa[k]:
            assert torch.equal(torch.as_tensor(sa[k][key]), torch.as_tensor(sb[k][key]))
    assert torch.equal(a.pos, b.pos)
    with pytest.raises(ValueError, match="already exists"):
        checkpoint.save(tmp_path / "ckpt", a)


def test_a_changed_file_is_refused(tmp_path: Path) -> None:
    a = _trainer(3)
    checkpoint.save(tmp_path / "ckpt", a)
    states = tmp_path / "ckpt" / "states.pt"
    states.write_bytes(states.read_bytes() + b"\0")
    with pytest.raises(ValueError, match="SHA-256"):
        checkpoint.restore(tmp_path / "ckpt", _trainer(4))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, root: str) -> None:
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = _trainer(10 + rank, distributed=True)
        for t in mine.state:  # this rank's rows carry values of their own
            if t.is_floating_point():
                t.add_(100.0 * rank)
        written = checkpoint.save(Path(root) / "dp", mine)
        assert (written is not None) == (rank == 0)
        dist.barrier()
        fresh = _trainer(20 + rank, distributed=True)
        checkpoint.restore(Path(root) / "dp", fresh)
        for x, y in zip(mine.state, fresh.state, strict=True):
            assert torch.equal(x, y), rank
    finally:
        dist.destroy_process_group()


def test_two_ranks_save_one_checkpoint_and_each_restores_its_own_rows(tmp_path: Path) -> None:
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    saved = torch.load(tmp_path / "dp" / "states.pt", weights_only=True)
    assert len(saved["groups"]) == 2 and saved["mixer"] is None
    layout = json.loads((tmp_path / "dp" / "train.json").read_text())["layout"]
    assert layout == {"groups": 2, "rows_per_group": B, "tokens_per_row": N}
