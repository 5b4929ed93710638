"""The loop and its halting on a B200 (the contract of ``vesper/loop.py`` of mstampfli/vesper-preview).

``T_max`` passes of ``C`` columns: pass ``t`` conditions the input with ``u_t``, runs every column
through its pass-``t`` state, and an exit rule decides which tokens halt (ACT by default:
accumulate ``p_t = sigmoid(w_h . RMSNorm(x) + b_h)``, halt at ``P + p >= 1 - epsilon``, output
the allocation-weighted mean of the pass outputs). A halted token leaves the active set and its
projections of its exit pass are copied forward into every later pass's states (``Carry``).

The arithmetic of the decision, the output weights and the counts is the reference's, operation
for operation, in torch (so pass counts agree to the bit on the same inputs); what changes is the
per-token bookkeeping around it. The reference's copy-forward merge (``vesper/loop.py:523-537``:
tokens halting now take their fresh projections, every other token keeps the previous ones) is
the column's written projections themselves: a column with a carry writes a halted token's
carried projections, so the merge changes only tokens still active, whose carried values no later
pass reads. The zeroing of halted rows and the selection of the next input are each one
multi-tensor select launch (``vb_select_rows``). With ``compact_rows`` (the default) every pass
after the first compacts the active tokens once (``compact_flat``) and the columns run every
per-token step on those rows only, as bucketed work that follows the live count on the device
(``vesper_b200.kernels.slabs``): the reference computes them densely and discards the halted
rows' outputs (``vesper/loop.py:24-26``).
"""

from __future__ import annotations

import math
from collections.abc import Callable, Sequence
from dataclasses import dataclass
from typing import Protocol

import torch
import torch.nn.functional as F  # noqa: N812
from torch import Tensor, nn
from torch.utils.checkpoint import checkpoint

from vesper_b200.column import Carry, Column, ColumnState, Projections, RMSNorm
from vesper_b200.contracts import ContractError, Dims, check_shape, require
from vesper_b200.kernels.compact import compact_flat, select_rows
from vesper_b200.kernels.slabs import SLAB_FIRST

CDF_SLACK = 1e-9  # vesper/exits.py:164
HAZARD_LIMIT = 1e4  # vesper/exits.py:234

ExitStep = Callable[..., tuple[Tensor, Tensor]]


class HaltingHead(nn.Module):
    """``sigmoid(w_h . RMSNorm(x) + b_h)`` (``vesper/loop.py:93-149``), the reference's draws."""

    def __init__(self, d: int, generator: torch.Generator | None = None) -> None:
        super().__init__()
        self.norm = RMSNorm(d)
        self.w_h = nn.Parameter(torch.randn(d, generator=generator) / math.sqrt(d))
        self.b_h = nn.Parameter(torch.zeros(()))

    def logit(self, x: Tensor, pass_index: int) -> Tensor:
        del pass_index
        return self.norm.forward(x) @ self.w_h + self.b_h

    def probability(self, x: Tensor, pass_index: int) -> Tensor:
        return torch.sigmoid(self.logit(x, pass_index))

    def forward(self, x: Tensor) -> Tensor:
        return self.probability(x, 0)


class ExitRule(Protocol):
    def begin(self, active: Tensor, dtype: torch.dtype, runs: int) -> ExitStep: ...


@dataclass(frozen=True)
class ActRule:
    """ACT (``vesper/loop.py:157-180``): ``a_t = p_t`` before the halting pass, ``1 - P`` at it."""

    halting: HaltingHead
    epsilon: float

    def begin(self, active: Tensor, dtype: torch.dtype, runs: int) -> ExitStep:
        del runs
        cumulative = torch.zeros(active.shape, dtype=dtype, device=active.device)

        def step(t: int, h: Tensor, active: Tensor, *, last: bool) -> tuple[Tensor, Tensor]:
            nonlocal cumulative
            p = torch.where(active, self.halting.probability(h, t), torch.zeros_like(cumulative))
            halts = active & ((cumulative + p >= 1.0 - self.epsilon) | last)
            allocation = torch.where(halts, 1.0 - cumulative, p)
            cumulative = cumulative + p
            return halts, allocation

        return step


@dataclass(frozen=True)
class DenseRule:
    """Every token runs every pass with fresh writes (``vesper/loop.py:183-200``)."""

    def begin(self, active: Tensor, dtype: torch.dtype, runs: int) -> ExitStep:
        del active, runs

        def step(t: int, h: Tensor, active: Tensor, *, last: bool) -> tuple[Tensor, Tensor]:
            del t, h
            halts = active & last
            return halts, halts.to(dtype)

        return step


@dataclass(frozen=True)
class TraceRule:
    """Exit every token at a given 1-based pass ``depths`` (``vesper/loop.py:203-241``)."""

    depths: Tensor

    def begin(self, active: Tensor, dtype: torch.dtype, runs: int) -> ExitStep:
        if self.depths.shape != active.shape:
            msg = f"trace of shape {tuple(self.depths.shape)} for tokens {tuple(active.shape)}"
            raise ContractError(msg)
        if self.depths.dtype not in {torch.int8, torch.int16, torch.int32, torch.int64}:
            msg = f"trace depths must be a signed integer tensor, got {self.depths.dtype}"
            raise ContractError(msg)
        if self.depths.numel():
            require(((self.depths >= 1) & (self.depths <= runs)).all(), f"trace depths must lie in [1, {runs}]")
        depths = self.depths.to(active.device)

        def step(t: int, h: Tensor, active: Tensor, *, last: bool) -> tuple[Tensor, Tensor]:
            del h
            halts = active & ((depths == t + 1) | last)
            return halts, halts.to(dtype)

        return step


def hazard_baseline(t_max: int, device: torch.device | None = None) -> Tensor:
    """``-log(T - t)`` for ``t = 1..T-1`` then 0, float64 (``vesper/exits.py:42-60``)."""
    if t_max < 1:
        msg = f"t_max must be at least 1, got {t_max}"
        raise ValueError(msg)
    passes = torch.arange(1, t_max, dtype=torch.float64, device=device)
    return torch.cat([-torch.log(t_max - passes), torch.zeros(1, dtype=torch.float64, device=device)])


@dataclass(frozen=True)
class CdfRule:
    """Exit at the first pass whose cumulative exit probability reaches ``q``
    (``vesper/loop.py:244-280`` with ``vesper/exits.py:167-194``), in float64."""

    head: HaltingHead | None
    q: float

    def begin(self, active: Tensor, dtype: torch.dtype, runs: int) -> ExitStep:
        if not 0.0 < self.q <= 1.0:
            msg = f"q must lie in (0, 1], got {self.q}"
            raise ValueError(msg)
        baseline = hazard_baseline(runs, active.device)
        survival = torch.zeros(active.shape, dtype=torch.float64, device=active.device)
        cdf = survival.clone()

        def step(t: int, h: Tensor, active: Tensor, *, last: bool) -> tuple[Tensor, Tensor]:
            nonlocal survival, cdf
            if not last:
                learned = (torch.zeros(active.shape, device=active.device) if self.head is None
                           else self.head.logit(h, t))  # fmt: skip
                z = (learned.to(torch.float64) + baseline[t]).clamp(-HAZARD_LIMIT, HAZARD_LIMIT)
                cdf = cdf + (F.logsigmoid(z) + survival).exp()
                survival = survival + F.logsigmoid(-z)
            halts = active & ((cdf >= self.q - CDF_SLACK) | last)
            return halts, halts.to(dtype)

        return step


@dataclass(frozen=True)
class LoopResult:
    """``y [b,n,d]``, the states, ``n_iters int32[b,n]``, ``ponder [b,n]``, ``per_pass [T,b,n,d]``."""

    y: Tensor
    states: tuple[ColumnState, ...]
    n_iters: Tensor
    ponder: Tensor
    per_pass: Tensor


class Loop(nn.Module):
    """``T_max`` passes of ``C`` columns with halting and copy-forward (``vesper/loop.py:300-465``)."""

    def __init__(self, columns: Sequence[Column], halting: HaltingHead, d: int, t_max: int, halt_epsilon: float) -> None:
        super().__init__()
        if len(columns) == 0:
            msg = "the loop needs at least one column"
            raise ValueError(msg)
        if t_max < 1:
            msg = f"t_max must be at least 1, got {t_max}"
            raise ValueError(msg)
        if not 0.0 < halt_epsilon < 1.0:
            msg = f"halt_epsilon must lie in (0, 1), got {halt_epsilon}"
            raise ValueError(msg)
        self.columns = tuple(columns)
        self.modules_ = nn.ModuleList(list(columns))
        self.halting = halting
        self.halting_module = halting
        self.t_max, self.halt_epsilon = t_max, halt_epsilon
        self.u = nn.Parameter(torch.zeros(t_max, d))
        self.compact_rows = True  # feed-forward blocks of passes after the first on active rows only

    def forward(self, x0: Tensor, pos: Tensor, states: Sequence[ColumnState], passes: int | None = None, *,
                recompute: bool = False, exit_rule: ExitRule | None = None,
                executed: int | None = None) -> LoopResult:  # fmt: skip
        """One chunk through the passes (``vesper/loop.py:349-465``), same arguments and errors."""
        runs = self.t_max if passes is None else passes
        if not 1 <= runs <= self.t_max:
            msg = f"passes must lie in [1, {self.t_max}], got {runs}"
            raise ValueError(msg)
        steps = runs if executed is None else executed
        if not 1 <= steps <= runs:
            msg = f"executed must lie in [1, {runs}], got {steps}"
            raise ValueError(msg)
        if len(states) != len(self.columns):
            msg = f"{len(states)} states for {len(self.columns)} columns"
            raise ValueError(msg)
        held = {self.t_max} if executed is None else {self.t_max, steps}
        for c, s in enumerate(states):
            counts = {len(s.h), len(s.kv), len(s.key_history)}
            if len(counts) != 1 or not counts <= held:
                msg = f"state of column {c} has {sorted(counts)} passes, the loop runs {self.t_max}"
                raise ValueError(msg)
        dims: Dims = {"d": self.u.shape[1]}
        check_shape("x0", x0, ("b", "n", "d"), dims)
        check_shape("pos", pos, ("b", "n"), dims, dtype=torch.long)
        b, n = dims["b"], dims["n"]
        device = x0.device
        active = torch.ones(b, n, dtype=torch.bool, device=device)
        rule = ActRule(self.halting, self.halt_epsilon) if exit_rule is None else exit_rule
        decide = rule.begin(active, x0.dtype, runs)
        dense = isinstance(rule, DenseRule)
        y = torch.zeros_like(x0)
        depth = torch.zeros(b, n, dtype=x0.dtype, device=device)
        n_iters = torch.zeros(b, n, dtype=torch.int32, device=device)
        carried: list[Projections | None] = [None] * len(self.columns)
        current = list(states)
        if executed is not None:
            current = [ColumnState(s.h[:steps], s.kv[:steps], s.key_history[:steps]) for s in states]
        x = x0
        per_pass: list[Tensor] = []
        for t in range(steps):
            h = x + self.u[t]
            fresh: list[Projections] = []
            rows = compact_flat(active, SLAB_FIRST) if self.compact_rows and t > 0 and not dense else None
            for c, column in enumerate(self.columns):
                previous = carried[c]
                carry = None if previous is None or dense else Carry(active, previous, rows)
                # with a carry the column zeroes the halted rows in its last residual add; without
                # one (the first pass) no token has halted yet
                if recompute:
                    h, current[c], written = checkpoint(column.step, h, pos, current[c], t, carry=carry,
                                                        zero_halted=True, use_reentrant=False)  # fmt: skip
                else:
                    h, current[c], written = column.step(h, pos, current[c], t, carry=carry, zero_halted=True)
                fresh.append(written)
                if not dense and carry is None and t > 0:
                    (h,) = select_rows(active, [h], [None])  # halted rows zeroed before anything reads them
            halts, allocation = decide(t, h, active, last=t == runs - 1)
            y = y + allocation[..., None] * h
            depth = depth + allocation * (t + 1)
            n_iters = n_iters + active.to(torch.int32)
            per_pass.append(h)
            if not dense:
                # the copy-forward merge: a halted token's written projections are its carried ones
                carried[:] = fresh
                (x,) = select_rows(active, [h], [x])
            else:
                x = h
            active = active & ~halts
        if steps < runs:
            require((~active).all(), f"every token must exit by executed pass {steps} of {runs}; the cap never forces")
        return LoopResult(y=y, states=tuple(current), n_iters=n_iters, ponder=depth, per_pass=torch.stack(per_pass))
