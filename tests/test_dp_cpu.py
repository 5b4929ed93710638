"""Data-parallel gradient exchange on the CPU: two ``gloo`` ranks, the bucket and its all-reduce.

``GradBucket`` keeps every ``.grad`` as a view into one flat float32 buffer, so a step's only
exchange is one all-reduce. Two processes (world size 2, ``gloo`` over 127.0.0.1) train a small
stand-in model on different rows; each checks that after backward the gradients still alias the
bucket, that the all-reduce left the average of both ranks' gradients (which each rank also
computes locally from both batches), that the clip follows ``clip_grad_norm_``'s rule, and that
the ranks end the optimizer step with identical parameters.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

from vesper_b200.train import GradBucket


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model() -> nn.Module:
    torch.manual_seed(0)
    return nn.Sequential(nn.Linear(16, 32), nn.Tanh(), nn.Linear(32, 4))


def _batch(rank: int) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator().manual_seed(100 + rank)
    return torch.randn(8, 16, generator=g), torch.randn(8, 4, generator=g)


def _worker(rank: int, world: int, port: int, out: dict) -> None:
    os.environ["MASTER_ADDR"], os.environ["MASTER_PORT"] = "127.0.0.1", str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = _model()
        params = list(model.parameters())
        bucket = GradBucket(params)
        # the average of both ranks' gradients, computed locally
        want = [torch.zeros_like(p) for p in params]
        for r in range(world):
            ref = _model()
            x, y = _batch(r)
            nn.functional.mse_loss(ref(x), y).backward()
            for w, p in zip(want, ref.parameters(), strict=True):
                w += p.grad / world
        bucket.zero()
        x, y = _batch(rank)
        nn.functional.mse_loss(model(x), y).backward()
        assert bucket.views_intact()
        bucket.allreduce()
        got = [p.grad.clone() for p in params]
        for g, w in zip(got, want, strict=True):
            torch.testing.assert_close(g, w, rtol=1e-6, atol=1e-7)
        norm_before = torch.cat([g.flatten() for g in got]).norm()
        norm = bucket.clip(0.01)
        torch.testing.assert_close(norm, norm_before)
        assert float(bucket.flat.norm()) <= 0.01 * (1 + 1e-5)
        opt = torch.optim.AdamW(params, lr=1e-2)
        opt.step()
        flat = torch.cat([p.detach().flatten() for p in params])
        gathered = [torch.zeros_like(flat) for _ in range(world)]
        dist.all_gather(gathered, flat)
        out[rank] = bool(torch.equal(gathered[0], gathered[1]))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_average_their_gradients_and_stay_in_step() -> None:
    ctx = mp.get_context("spawn")
    with ctx.Manager() as manager:
        out = manager.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=120)
        codes = [p.exitcode for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        assert codes == [0, 0], codes
        assert dict(out) == {0: True, 1: True}


def test_the_bucket_refuses_non_float32_parameters() -> None:
    with pytest.raises(ValueError, match="float32"):
        GradBucket([nn.Parameter(torch.zeros(3, dtype=torch.float64))])
