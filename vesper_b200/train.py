"""The training step on a B200, captured as one CUDA graph, data-parallel over NCCL.

The step of ``vesper/train.py:748-831`` (``_device_step``) for one chunk group: autocast-bf16
forward of the looped model with activation recomputation, the wake objective, backward, one
gradient clip, a capturable AdamW with the reference's decay roles (``vesper/train.py:93-124,
343-385``), and the carried per-pass states written back for the next chunk. ``TrainStep`` warms it
up eagerly on a side stream and captures it (``vesper/graphs.py:49-120``: ``CapturedStep``), so a
step is one graph replay.

Data parallel (one process per GPU, ``torch.distributed`` with NCCL): the gradients live in one
flat float32 bucket (each parameter's ``.grad`` is a view into it), so the only exchange of a step
is one all-reduce of that bucket, captured in the graph with the rest; each rank trains on its
own batch rows (weak scaling) and the clip sees the averaged gradient, as one process with the
whole batch would. The reference trains on one device; this is the north star's addition.
"""

from __future__ import annotations

from collections.abc import Sequence
from contextlib import contextmanager
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
from torch import Tensor, nn

from vesper_b200.column import ColumnShape, ColumnState, set_scan, state_tensors, with_state_tensors
from vesper_b200.model import Vesper

# weight-decay roles (vesper/train.py:93-124): decayed linear maps, undecayed gates, norms and u
DECAYED = frozenset({"embedding.weight", "rec.w_q", "rec.w_k", "rec.w_v", "rec.w_o", "attn.w_q", "attn.w_k",
                     "attn.w_v", "attn.w_o", "ffn.w1", "ffn.w2"})  # fmt: skip
UNDECAYED = frozenset({"rec.w_beta", "rec.conv_k", "halting.w_h", "halting.b_h", "halting.norm.weight", "loop.u",
                       "norm_rec.weight", "norm_attn.weight", "norm_ffn.weight", "norm_out.weight"})  # fmt: skip


@dataclass(frozen=True)
class StepConfig:
    """The model geometry and the optimizer recipe of one training step."""

    shape: ColumnShape
    vocab: int
    columns: int
    t_max: int
    halt_epsilon: float = 0.01
    lr: float = 3e-4
    betas: tuple[float, float] = (0.9, 0.95)
    weight_decay: float = 0.1
    grad_clip: float = 1.0
    lambda_h: float = 0.01
    recompute: bool = True
    slices: int = 8


# the looped d512 model of the train-step benchmark: 13 columns, 8 passes, 32k vocabulary
VESPER_S = StepConfig(
    shape=ColumnShape(d=512, heads=8, kv_groups=4, head_dim=64, window=512, rotary_base=10000.0, ffn_mult=3,
                      block=64, key_conv=4),  # fmt: skip
    vocab=32000, columns=13, t_max=8,
)


def decays(name: str) -> bool:
    """Whether parameter ``name`` takes weight decay, by its role (``vesper/train.py:343-354``)."""
    if any(name == r or name.endswith("." + r) for r in DECAYED):
        return True
    if any(name == r or name.endswith("." + r) for r in UNDECAYED):
        return False
    msg = f"parameter {name!r} has no weight-decay role; add it to DECAYED or UNDECAYED"
    raise ValueError(msg)


def unique_named_parameters(model: nn.Module) -> list[tuple[str, nn.Parameter]]:
    return list(model.named_parameters())  # shared parameters appear once


class GradBucket:
    """Every parameter's gradient as a view into one flat float32 buffer (one all-reduce)."""

    def __init__(self, params: Sequence[nn.Parameter]) -> None:
        self.params = list(params)
        total = sum(p.numel() for p in self.params)
        dev = self.params[0].device
        self.flat = torch.zeros(total, dtype=torch.float32, device=dev)
        offset = 0
        for p in self.params:
            if p.dtype != torch.float32:
                msg = f"gradient bucket: parameters are float32, got {p.dtype}"
                raise ValueError(msg)
            p.grad = self.flat[offset : offset + p.numel()].view_as(p)
            offset += p.numel()

    def zero(self) -> None:
        self.flat.zero_()

    def views_intact(self) -> bool:
        """Whether every ``.grad`` still aliases the bucket (autograd accumulated in place)."""
        base = self.flat.data_ptr()
        end = base + self.flat.numel() * 4
        return all(p.grad is not None and base <= p.grad.data_ptr() < end for p in self.params)

    def allreduce(self, group: dist.ProcessGroup | None = None) -> None:
        """Average the gradients over the group's ranks (NCCL on CUDA, gloo on the CPU)."""
        dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=group)
        self.flat.div_(dist.get_world_size(group))

    def clip(self, max_norm: float) -> Tensor:
        """Scale to an L2 norm of at most ``max_norm`` (``clip_grad_norm_``'s rule); the norm before."""
        norm = self.flat.norm()
        self.flat.mul_(torch.clamp(max_norm / (norm + 1e-6), max=1.0))
        return norm


def optimizer(model: nn.Module, cfg: StepConfig) -> torch.optim.AdamW:
    """Capturable AdamW, two groups by role, the rate a device tensor (``vesper/train.py:357-385``)."""
    named = unique_named_parameters(model)
    decayed = [p for n, p in named if decays(n)]
    plain = [p for n, p in named if not decays(n)]
    dev = named[0][1].device
    lr = torch.tensor(cfg.lr, device=dev)
    groups = [{"params": decayed, "weight_decay": cfg.weight_decay}, {"params": plain, "weight_decay": 0.0}]
    return torch.optim.AdamW(groups, lr=lr, betas=cfg.betas, capturable=True, foreach=True)


@contextmanager
def side_stream():
    """Eager warm-up steps on a fresh stream joined to the current one (``vesper/graphs.py:41-47``)."""
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        yield
    torch.cuda.current_stream().wait_stream(stream)


@dataclass
class TrainStep:
    """One training step over ``b`` rows of ``n`` tokens, captured after ``warm`` eager steps.

    ``load(tokens, targets, mask)`` copies a batch into the static inputs; ``run()`` replays (or,
    before the capture, runs eagerly) and returns ``[loss, ntp, ponder, grad_norm, n_iters]``, the
    tensors overwritten by the next step. The per-pass states carry from step to step inside the
    graph (the stream's next chunk), positions advance by ``n`` per step.
    """

    model: Vesper
    cfg: StepConfig
    b: int
    n: int
    group: dist.ProcessGroup | None = None
    distributed: bool = False
    warm: int = 3
    graph: torch.cuda.CUDAGraph | None = field(default=None, init=False)

    def __post_init__(self) -> None:
        dev = next(self.model.parameters()).device
        self.device = dev
        set_scan(self.model, "fused")
        self.params = [p for _, p in unique_named_parameters(self.model)]
        self.bucket = GradBucket(self.params)
        self.opt = optimizer(self.model, self.cfg)
        self.tokens = torch.zeros(self.b, self.n, dtype=torch.long, device=dev)
        self.targets = torch.zeros(self.b, self.n, dtype=torch.long, device=dev)
        self.mask = torch.ones(self.b, self.n, dtype=torch.bool, device=dev)
        self.pos = torch.arange(self.n, device=dev).expand(self.b, self.n).contiguous()
        self.templates: list[ColumnState] = self.model.init_states(self.b, torch.bfloat16, dev)
        self.state = state_tensors(self.templates)
        self.steps = 0
        self.filled = False  # the attention windows have their steady shape (after the first chunk)
        self.outputs: list[Tensor] | None = None

    def adopt_states(self, states: list[ColumnState]) -> None:
        """Take steady-state carried states (a restored checkpoint's) before the first step."""
        if self.graph is not None:
            msg = "the step is captured: carried states can only be copied into it"
            raise ValueError(msg)
        self.templates = [_detached(s) for s in states]
        self.state = [t.to(self.device).clone() for t in state_tensors(self.templates)]
        self.templates = with_state_tensors(self.templates, self.state)
        self.filled = True

    def load(self, tokens: Tensor, targets: Tensor, mask: Tensor | None = None) -> None:
        self.tokens.copy_(tokens, non_blocking=True)
        self.targets.copy_(targets, non_blocking=True)
        if mask is not None:
            self.mask.copy_(mask, non_blocking=True)

    def _body(self) -> list[Tensor]:
        self.bucket.zero()
        states = with_state_tensors(self.templates, self.state)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            result = self.model.run(self.tokens, self.pos, states, recompute=self.cfg.recompute)
            total, parts = self.model.objective(result, self.targets, self.mask, self.cfg.lambda_h, self.cfg.slices)
        total.backward()
        if self.distributed:
            self.bucket.allreduce(self.group)
        norm = self.bucket.clip(self.cfg.grad_clip)
        self.opt.step()
        new = state_tensors([_detached(s) for s in result.states])
        for old, fresh in zip(self.state, new, strict=True):
            old.copy_(fresh)
        self.pos.add_(self.n)
        return [total.detach(), parts["ntp"].detach(), parts["ponder"].detach(), norm, result.n_iters]

    def _eager(self) -> list[Tensor]:
        if not self.filled:
            # the first chunk fills the attention windows: afterwards every state has its steady
            # shape, which the static state tensors (and the capture) take
            self.bucket.zero()
            states = with_state_tensors(self.templates, self.state)
            out = self._first(states)
            return out
        with side_stream():
            return self._body()

    def _first(self, states: list[ColumnState]) -> list[Tensor]:
        with torch.autocast("cuda", dtype=torch.bfloat16):
            result = self.model.run(self.tokens, self.pos, states, recompute=self.cfg.recompute)
            total, parts = self.model.objective(result, self.targets, self.mask, self.cfg.lambda_h, self.cfg.slices)
        total.backward()
        if self.distributed:
            self.bucket.allreduce(self.group)
        norm = self.bucket.clip(self.cfg.grad_clip)
        self.opt.step()
        self.templates = [_detached(s) for s in result.states]
        self.state = [t.clone() for t in state_tensors(self.templates)]
        self.filled = True
        self.pos.add_(self.n)
        return [total.detach(), parts["ntp"].detach(), parts["ponder"].detach(), norm, result.n_iters]

    def run(self) -> list[Tensor]:
        """One step: eager while warming up, then one capture, then replays."""
        if self.steps < self.warm:
            out = self._eager()
        else:
            if self.graph is None:
                torch.cuda.synchronize()
                self.graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(self.graph):
                    self.outputs = self._body()
            self.graph.replay()
            out = self.outputs
        self.steps += 1
        assert self.bucket.views_intact(), "a gradient left the bucket"
        return out

    def save(self, path) -> object:
        """Write a checkpoint (``vesper_b200.checkpoint.save``; every rank calls it)."""
        from vesper_b200 import checkpoint  # noqa: PLC0415

        return checkpoint.save(path, self)

    def restore(self, path) -> dict[str, object]:
        """Load a checkpoint in place (``vesper_b200.checkpoint.restore``)."""
        from vesper_b200 import checkpoint  # noqa: PLC0415

        return checkpoint.restore(path, self)

    def release(self) -> None:
        """Drop the graph (it holds the NCCL all-reduce) before the process group goes."""
        self.graph = None
        self.outputs = None


def _detached(state: ColumnState) -> ColumnState:
    from vesper_b200.column import map_state  # noqa: PLC0415

    return map_state(state, lambda t: t.detach())
