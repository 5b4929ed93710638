"""The captured training step on a B200: replays equal the eager steps bit for bit.

The step of vesper/train.py:748-831 (forward with recomputation, objective, backward, clip,
capturable AdamW, carried states) on a small looped model: one ``TrainStep`` stays eager for six
steps, a second one, built from the same seed, captures at its fourth step and replays. Losses,
gradient norms, pass counts and every parameter after the six steps must be identical (the
reference's own bar, tests/test_train_graph.py: captured == eager bitwise), and the loss must fall
on a repeated batch (the step trains).
"""

from __future__ import annotations

import pytest
import torch

from vesper_b200 import _lib
from vesper_b200.column import ColumnShape
from vesper_b200.model import Vesper
from vesper_b200.train import StepConfig, TrainStep

pytestmark = pytest.mark.gpu
CUDA = torch.device("cuda")
CFG = StepConfig(
    shape=ColumnShape(d=64, heads=2, kv_groups=2, head_dim=32, window=16, rotary_base=10000.0, ffn_mult=2,
                      block=16, key_conv=4),  # fmt: skip
    vocab=97, columns=2, t_max=3, lr=3e-3, slices=2,
)


def _trainer(warm: int) -> TrainStep:
    model = Vesper(CFG.shape, CFG.vocab, CFG.columns, CFG.t_max, CFG.halt_epsilon, torch.Generator().manual_seed(3))
    return TrainStep(model.to(CUDA), CFG, b=2, n=48, warm=warm)


def _batch():
    g = torch.Generator().manual_seed(4)
    tokens = torch.randint(0, CFG.vocab, (2, 49), generator=g)
    return tokens[:, :-1].to(CUDA), tokens[:, 1:].to(CUDA)


def test_captured_steps_replay_the_eager_steps_bitwise_and_train() -> None:
    tokens, targets = _batch()
    runs = []
    for warm in (100, 3):
        trainer = _trainer(warm)
        outs = []
        for _ in range(6):
            trainer.load(tokens, targets)
            outs.append([t.clone() for t in trainer.run()])
        torch.cuda.synchronize()
        _lib.check_status(CUDA)
        runs.append((outs, [p.detach().clone() for p in trainer.params]))
        assert (trainer.graph is None) == (warm == 100)
        trainer.release()
    (eager, p_eager), (captured, p_captured) = runs
    for step, (a, b) in enumerate(zip(eager, captured, strict=True)):
        for x, y in zip(a, b, strict=True):
            assert torch.equal(x, y), step
    assert all(torch.equal(a, b) for a, b in zip(p_eager, p_captured, strict=True))
    losses = [float(o[0]) for o in eager]
    assert losses[-1] < losses[0], losses
