"""Batched one-token decoding of the looped model on a B200, captured as one CUDA graph.

The contract of ``vesper/decode.py`` (``decode_step`` ``:29-46``, ``CapturedDecoder`` ``:49-97``)
of mstampfli/vesper-preview, batched: the reference decoder takes one row (its ring writes one
slot per row); here every row of a batch decodes its own stream in the same step. A step embeds
one token per row, runs the loop at a fixed depth with every token active in every pass (the
reference's ``DenseRule``: ``y`` is the last pass's output), applies the head to it and takes the
argmax over the first ``vocab`` ids. Every column keeps, per pass, its float32 recurrent state,
its key history and a ``RingKVCache``; the step updates all of them IN PLACE (``Column.step_decode``:
the one-token scan kernel, the batched ring-attention kernel), so their shapes and addresses never
change and one captured graph serves every step.

``prefill`` is the long-context half: the prompt runs through the ordinary chunked forward
(``Vesper.run`` with the dense rule, chronological ``KVCache`` windows, the chunked scan and
window-attention kernels), chunk by chunk with carried states, and its windows are then moved into
rings (``ring_from_cache``), so decoding continues exactly where the prompt ended.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch
from torch import Tensor

from vesper_b200.attention import ring_from_cache
from vesper_b200.column import ColumnState, state_tensors
from vesper_b200.contracts import ContractError
from vesper_b200.loop import DenseRule
from vesper_b200.model import Vesper


def decode_forward(model: Vesper, token: Tensor, position: Tensor, states: Sequence[ColumnState], depth: int) -> Tensor:
    """``y [b, 1, d]`` of one token per row at ``depth`` dense passes, states updated in place.

    The loop of ``vesper/loop.py:349-465`` under ``DenseRule`` (every token active in every pass;
    the output is the last pass's) for ``n = 1``.
    """
    x = model.embedding.embed(token)
    for t in range(depth):
        h = x + model.loop.u[t]
        for c, column in enumerate(model.loop.columns):
            h = column.step_decode(h, position, states[c], t)
        x = h
    return x


def decode_step(model: Vesper, depth: int, vocab: int, states: Sequence[ColumnState], token: Tensor,
                position: Tensor) -> tuple[Tensor, Tensor]:  # fmt: skip
    """``(ids [b, 1], logits [b, 1, vocab])`` of one token per row (``vesper/decode.py:29-46``),
    the states advanced in place."""
    y = decode_forward(model, token, position, states, depth)
    logits = model.head(y)[..., :vocab]
    return logits.argmax(-1), logits


class BatchedDecoder:
    """Greedy decoding of ``b`` rows at ``depth`` passes, the step captured after ``warm`` eager steps.

    ``prefill(tokens)`` runs a prompt ``[b, P]`` (positions ``0 .. P-1``) and returns the logits of
    every prompt position; ``step(token)`` advances every row by one token ``[b, 1]`` at the next
    position and returns ``(ids, logits)`` (the graph's buffers after a replay: read them before the
    next step). ``dtype``: the activation dtype (bfloat16 runs under autocast with the chunked and
    one-token bf16 kernels; float32 is the reference's precision).

    Raises:
        ContractError: if the model is not on CUDA or ``depth`` is outside ``1..t_max``.
    """

    def __init__(self, model: Vesper, depth: int, vocab: int, b: int, dtype: torch.dtype = torch.bfloat16,
                 warm: int = 2) -> None:  # fmt: skip
        device = next(model.parameters()).device
        if device.type != "cuda":
            msg = f"the decoder runs on CUDA, the model is on {device}"
            raise ContractError(msg)
        if not 1 <= depth <= model.t_max:
            msg = f"depth {depth} is outside 1..{model.t_max}"
            raise ContractError(msg)
        self.model, self.depth, self.vocab, self.b, self.dtype, self.warm = model, depth, vocab, b, dtype, warm
        self.device = device
        self.states: list[ColumnState] = model.init_states(b, dtype, device, ring=True)
        self.token = torch.zeros(b, 1, dtype=torch.long, device=device)
        self.position = torch.zeros(b, 1, dtype=torch.long, device=device)
        self.graph: torch.cuda.CUDAGraph | None = None
        self.outputs: tuple[Tensor, Tensor] | None = None
        self.steps = 0

    def _autocast(self):
        return torch.autocast("cuda", dtype=torch.bfloat16, enabled=self.dtype == torch.bfloat16)

    @torch.no_grad()
    def prefill(self, tokens: Tensor, chunk: int = 2048, *, all_logits: bool = False) -> Tensor:
        """Run the prompt ``[b, P]`` chunk by chunk; the rings then hold its last windows.

        Returns the logits of the last prompt position ``[b, 1, vocab]`` (of every position with
        ``all_logits``, ``[b, P, vocab]``: a long prompt's full logits are large)."""
        b, length = tokens.shape
        if b != self.b:
            msg = f"prompt of {b} rows for a decoder of {self.b}"
            raise ContractError(msg)
        states = self.model.init_states(b, self.dtype, self.device)
        outs = []
        for s in range(0, length, chunk):
            piece = tokens[:, s : s + chunk].to(self.device)
            pos = torch.arange(s, s + piece.shape[1], device=self.device).expand(b, -1).contiguous()
            with self._autocast():
                res = self.model.run(piece, pos, states, passes=self.depth, exit_rule=DenseRule())
                if all_logits or s + chunk >= length:
                    outs.append(self.model.head(res.y if all_logits else res.y[:, -1:])[..., : self.vocab])
            states = list(res.states)
        rings = [ColumnState(h=s.h, kv=tuple(ring_from_cache(c) for c in s.kv), key_history=s.key_history)
                 for s in states]  # fmt: skip
        # into the decoder's own (possibly captured) buffers
        for dst, src in zip(state_tensors(self.states), state_tensors(rings), strict=True):
            dst.copy_(src)
        self.position.fill_(length - 1)
        return torch.cat(outs, dim=1)

    def _body(self) -> tuple[Tensor, Tensor]:
        self.position.add_(1)
        with self._autocast():
            return decode_step(self.model, self.depth, self.vocab, self.states, self.token, self.position)

    @torch.no_grad()
    def step(self, token: Tensor) -> tuple[Tensor, Tensor]:
        """One token per row ``[b, 1]`` at the next position: ``(ids [b, 1], logits [b, 1, vocab])``."""
        self.token.copy_(token)
        if self.steps < self.warm:  # eager, on a side stream joined to the current one
            side = torch.cuda.Stream(self.device)
            side.wait_stream(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(side):
                out = self._body()
            torch.cuda.current_stream(self.device).wait_stream(side)
        else:
            if self.graph is None:
                # capturing records the step without running it: the live buffers are untouched
                torch.cuda.synchronize(self.device)
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph):
                    self.outputs = self._body()
            self.graph.replay()
            out = self.outputs
        self.steps += 1
        return out

    def release(self) -> None:
        self.graph = None
        self.outputs = None

