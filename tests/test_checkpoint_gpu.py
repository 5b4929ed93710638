"""Resuming the captured training step from a checkpoint on a B200.

A ``TrainStep`` trains a small looped model for three steps (two eager, then the capture and a
replay), writes a checkpoint (weights, the capturable AdamW's state, the carried per-pass states and
the stream position) and trains two more steps. A second trainer built from another seed restores
the checkpoint and trains the same two steps: its losses, pass counts and final parameters equal the
uninterrupted run's bit for bit (a resumed run continues exactly where the saved one stood).
"""

from __future__ import annotations

from pathlib import Path

import pytest
import torch

from vesper_b200.column import ColumnShape
from vesper_b200.model import Vesper
from vesper_b200.train import StepConfig, TrainStep

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")
SHAPE = ColumnShape(d=64, heads=2, kv_groups=2, head_dim=32, window=32, rotary_base=10000.0, ffn_mult=2,
                    block=16, key_conv=4)  # fmt: skip
CFG = StepConfig(shape=SHAPE, vocab=256, columns=2, t_max=3)
B, N = 2, 64


def _trainer(seed: int) -> TrainStep:
    model = Vesper(SHAPE, CFG.vocab, CFG.columns, CFG.t_max, CFG.halt_epsilon, torch.Generator().manual_seed(seed))
    return TrainStep(model.to(CUDA), CFG, b=B, n=N, warm=2)


def _batches() -> list[torch.Tensor]:
    g = torch.Generator(device=CUDA).manual_seed(5)
    return [torch.randint(0, CFG.vocab, (B, N + 1), device=CUDA, generator=g) for _ in range(5)]


def _step(tr: TrainStep, batch: torch.Tensor) -> list[torch.Tensor]:
    tr.load(batch[:, :-1], batch[:, 1:])
    return [t.clone() for t in tr.run()]


def test_a_restored_trainer_continues_bit_for_bit(tmp_path: Path) -> None:
    batches = _batches()
    a = _trainer(0)
    for i in range(3):
        _step(a, batches[i])
    a.save(tmp_path / "ckpt")
    want = [_step(a, batches[i]) for i in (3, 4)]
    b = _trainer(1)
    b.restore(tmp_path / "ckpt")
    got = [_step(b, batches[i]) for i in (3, 4)]
    for w, g in zip(want, got, strict=True):
        for x, y in zip(w, g, strict=True):
            assert torch.equal(x, y), (x, y)
    for (name, p), q in zip(a.model.named_parameters(), b.model.parameters(), strict=True):
        assert torch.equal(p, q), name
    a.release()
    b.release()
