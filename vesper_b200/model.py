"""The model around the loop (the contract of ``vesper/model.py`` and ``vesper/embedding.py`` of
mstampfli/vesper-preview): tied embedding, the loop of columns, final norm, tied head, the wake
objective (mean next-token loss over the loss positions plus ``lambda_h`` times the mean ponder).

Same parameters and initialization draws as the reference's ``Vesper`` (embedding, then the
columns, then the halting head), so its ``state_dict`` loads. The head's loss is ``linear_nll``
per slice of positions (the reference's fused head: cuBLAS matmuls around this library's row
kernels, no float32 vocabulary logits); the objective keeps static shapes (every position is
scored, the ones outside the mask are replaced before the head), so the step can be captured.
"""

from __future__ import annotations

import math
from collections.abc import Sequence

import torch
import torch.nn.functional as F  # noqa: N812
from torch import Tensor, nn

from vesper_b200.column import Column, ColumnShape, ColumnState, RMSNorm, init_column_state
from vesper_b200.contracts import Dims, check_ids, check_shape
from vesper_b200.kernels.nll import linear_nll
from vesper_b200.loop import ExitRule, HaltingHead, Loop, LoopResult


class TiedEmbedding(nn.Module):
    """One matrix ``E [V, d]``: ``embed`` looks rows up, ``logits`` projects onto it."""

    def __init__(self, vocab: int, d: int, generator: torch.Generator | None = None) -> None:
        super().__init__()
        if vocab < 1 or d < 1:
            msg = f"vocab ({vocab}) and d ({d}) must be at least 1"
            raise ValueError(msg)
        self.vocab, self.d = vocab, d
        self.weight = nn.Parameter(torch.randn(vocab, d, generator=generator) / math.sqrt(d))

    def embed(self, tokens: Tensor) -> Tensor:
        return F.embedding(check_ids("tokens", tokens, ("b", "n"), {}, self.vocab), self.weight)

    def logits(self, x: Tensor) -> Tensor:
        return F.linear(x, self.weight)


class Vesper(nn.Module):
    """Embedding, loop, final norm and head (``vesper/model.py:42-132``)."""

    def __init__(self, shape: ColumnShape, vocab: int, columns: int, t_max: int, halt_epsilon: float,
                 generator: torch.Generator | None = None) -> None:  # fmt: skip
        super().__init__()
        self.embedding = TiedEmbedding(vocab, shape.d, generator)
        cols = [Column(shape, generator) for _ in range(columns)]
        self.loop = Loop(cols, HaltingHead(shape.d, generator), shape.d, t_max, halt_epsilon)
        self.norm_out = RMSNorm(shape.d)
        self.shape, self.columns, self.t_max = shape, columns, t_max

    def init_states(self, b: int, dtype: torch.dtype, device: torch.device, *, ring: bool = False) -> list[ColumnState]:
        return [init_column_state(self.shape, b, self.t_max, dtype, device, ring=ring) for _ in range(self.columns)]

    def head(self, y: Tensor) -> Tensor:
        """Outputs ``[b, n, d]`` to logits ``[b, n, V]``: the output norm, then the tied embedding
        (``vesper/model.py:128-141``)."""
        return self.embedding.logits(self.norm_out.forward(y))

    def run(self, tokens: Tensor, pos: Tensor, states: Sequence[ColumnState], passes: int | None = None, *,
            recompute: bool = False, exit_rule: ExitRule | None = None) -> LoopResult:  # fmt: skip
        return self.loop.forward(self.embedding.embed(tokens), pos, states, passes, recompute=recompute,
                                 exit_rule=exit_rule)  # fmt: skip

    def objective(self, result: LoopResult, targets: Tensor, mask: Tensor, lambda_h: float | Tensor,
                  slices: int = 1) -> tuple[Tensor, dict[str, Tensor]]:  # fmt: skip
        """``ntp + lambda_h * ponder`` over the positions ``mask`` marks (``vesper/model.py:141-181``)."""
        dims: Dims = {}
        check_shape("targets", targets, ("b", "n"), dims)
        check_shape("mask", mask, ("b", "n"), dims, dtype=torch.bool)
        b, n, d = result.y.shape
        keep = mask.reshape(b * n)
        rows = torch.where(keep[:, None], result.y.reshape(b * n, d), 0.0)
        tgt = torch.where(mask, targets, 0).reshape(b * n)
        width = -(-(b * n) // max(slices, 1))
        summed = torch.zeros((), dtype=torch.float32, device=rows.device)
        for s in range(0, b * n, width):
            losses = token_losses(self, rows[s : s + width], tgt[s : s + width])
            summed = summed + torch.where(keep[s : s + width], losses, 0.0).sum()
        count = mask.sum()
        ntp = summed / count
        ponder = torch.where(mask, result.ponder, 0.0).sum() / count
        total = ntp + lambda_h * ponder
        return total, {"ntp": ntp, "ponder": lambda_h * ponder}


def token_losses(model: Vesper, y: Tensor, targets: Tensor, *, keep_logits: bool = False) -> Tensor:
    """Per-token losses ``[...]`` of positions ``y [..., d]`` through the head
    (``vesper/model.py:314-342``): the head's norm, then ``linear_nll`` over the tied embedding,
    which keeps no float32 vocabulary logits."""
    lead = tuple(f"lead{i}" for i in range(y.dim() - 1))
    dims: Dims = {}
    check_shape("y", y, (*lead, "d"), dims)
    check_shape("targets", targets, lead, dims)
    x = model.norm_out.forward(y.reshape(1, -1, y.shape[-1]))[0]
    losses = linear_nll(x, model.embedding.weight, targets.reshape(-1), keep_logits=keep_logits)
    return losses.view(targets.shape)


def count_parameters(model: nn.Module) -> int:
    return sum(p.numel() for p in model.parameters())
