"""Benchmark of the vesper-b200 hot path: config 2 of BASELINE.json on B200s.

One step = the fused key pipeline + RMSNorm + bf16 delta scan, forward and backward, on
B=8, H=8, T=4096, d=128 (width 1024): ``x -> fused_rms_norm -> fused_keys -> delta_scan_fused``
with q, v, beta and the upstream gradient as further inputs, then the backward through all three
(gradients of x, the gain, the taps, q, v and beta). Synthetic inputs with the config's
distributions. Inputs are far larger than L2 (about 1 GB per step), so no flush is needed.

A second leg times config 4, the looped d512 model's training step (13 columns x 8 passes with ACT
halting and copy-forward, B=32 x T=2048 per GPU, activation recomputation, clip, AdamW), captured
as one CUDA graph, data-parallel with one NCCL all-reduce of the gradient bucket per step; it is
reported under ``train_step`` in the same line (``--no-train`` skips it).

Usage: ``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]``; for N > 1
it is launched by torchrun, one rank per GPU, each rank running the same per-GPU workload on its own
(batch x head) units with no collective on the data path (weak scaling); the time is the maximum
over ranks. ``--impl reference`` times the reference's CPU path (the float64 C restatement in
``oracle/``, all host threads) on a bounded sample of the same workload, on rank 0 only.

Prints one JSON line (rank 0).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "delta-scan fwd+bwd tokens/s/GPU & % roofline; vesper-s train tokens/s at 1/2/4/8 GPU"
B, H, T, D = 8, 8, 4096, 128
WIDTH = H * D
TAPS = 4
WORKLOAD = (
    "config 2: RMSNorm(width 1024) -> causal key filter (K=4) + L2 norm -> bf16 delta scan, "
    "forward+backward, B=8 H=8 T=4096 d=128"
)


def peaks() -> dict:
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text())
    except (OSError, ValueError):
        return {}


def scan_algorithmic_bytes(b: int, t: int, h: int, d: int) -> int:
    """HBM bytes the delta-scan fwd+bwd must move: (22d+6) per token-head + 5 state passes."""
    return b * t * h * (22 * d + 6) + b * h * 5 * 4 * d * d


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons while the timed region runs."""

    FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu: str) -> None:
        self.gpu = gpu
        self.proc: subprocess.Popen | None = None

    def __enter__(self) -> Clocks:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )  # fmt: skip
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc: object) -> None:
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        else:
            self.lines = []

    def summary(self) -> dict:
        sms, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9], strict=True):
                if flag.lower() == "active":
                    reasons.add(name)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {
            "sm_mhz": statistics.median(sms),
            "sm_max_mhz": max(maxes),
            "reasons": sorted(reasons),
            "samples": len(sms),
        }


def _gpu_id(device, local: int) -> str:
    """The nvidia-smi id of ``device`` (its UUID when torch reports one)."""
    import torch

    uuid = getattr(torch.cuda.get_device_properties(device), "uuid", None)
    if uuid:
        text = str(uuid)
        return text if text.startswith("GPU-") else f"GPU-{text}"
    return str(local)


def make_inputs(device, seed: int):
    import torch

    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(B, T, WIDTH, device=device, generator=g).bfloat16()
    q = torch.nn.functional.normalize(torch.randn(B, T, H, D, device=device, generator=g), dim=-1).bfloat16()
    v = torch.randn(B, T, H, D, device=device, generator=g).bfloat16()
    beta = torch.sigmoid(torch.randn(B, T, H, device=device, generator=g)).bfloat16()
    d_o = torch.randn(B, T, H, D, device=device, generator=g).bfloat16()
    taps = 0.5 * torch.randn(TAPS, WIDTH, device=device, generator=g)
    gain = torch.ones(WIDTH, device=device)
    hist = torch.zeros(B, TAPS - 1, WIDTH, device=device)
    s0 = torch.zeros(B, H, D, D, device=device)
    return {"x": x, "q": q, "v": v, "beta": beta, "d_o": d_o, "taps": taps, "gain": gain, "hist": hist, "s0": s0}


def step(inp, leaves):
    """One forward+backward through the public entry points; returns the outputs and gradients."""
    import torch

    from vesper_b200.kernels.delta_scan import delta_scan_fused
    from vesper_b200.kernels.keys import fused_keys
    from vesper_b200.kernels.norm import fused_rms_norm

    x, q, v, beta, gain, taps = leaves
    xn = fused_rms_norm(x, gain, 1e-3, 1e-6)
    k = fused_keys(xn, inp["hist"], taps, H)
    o, _ = delta_scan_fused(q, k, v, beta, inp["s0"])
    grads = torch.autograd.grad([o], [x, q, v, beta, gain, taps], [inp["d_o"]])
    return o, grads


def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from vesper_b200 import _lib
    from vesper_b200.kernels.delta_scan import check_status, scan_bf16_backward, scan_bf16_forward

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    inp = make_inputs(device, seed=1234 + rank)
    leaves = [inp[n].detach().requires_grad_() for n in ("x", "q", "v", "beta", "gain", "taps")]
    if args.profile_step:
        # one eager step after warm-up, for an ncu capture of each kernel once at full size
        for _ in range(max(args.warmup, 1)):
            step(inp, leaves)
        torch.cuda.synchronize(device)
        step(inp, leaves)
        torch.cuda.synchronize(device)
        check_status(device)
        return

    # --- device-resident throughput: the step captured once, replayed K times -----------------
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(3):
            step(inp, leaves)
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    check_status(device)
    graph = torch.cuda.CUDAGraph()
    before = _lib.launch_count()
    with torch.cuda.graph(graph):
        step(inp, leaves)
    launches_per_step = _lib.launch_count() - before
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize(device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(_gpu_id(device, local)) as clocks:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)
        start.record()
        for _ in range(args.steps):
            graph.replay()
        stop.record()
        torch.cuda.synchronize(device)
        if world > 1:
            dist.barrier()
    elapsed_ms = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([elapsed_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    check_status(device)
    tokens = world * B * T * args.steps
    value = tokens / (elapsed_ms / 1e3)
    del graph

    # --- roofline of the dominant kernel group: delta-scan fwd+bwd, CUDA events on its stream ---
    q, k, v, beta, s0 = inp["q"], inp["x"].view(B, T, H, D), inp["v"], inp["beta"], inp["s0"]
    k = torch.nn.functional.normalize(k.float(), dim=-1).bfloat16()
    _, _, saved = scan_bf16_forward(q, k, v, beta, s0)
    reps = max(5, min(args.steps, 50))
    for _ in range(3):
        scan_bf16_forward(q, k, v, beta, s0)
        scan_bf16_backward(q, k, v, beta, saved, inp["d_o"], None)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        _, _, saved = scan_bf16_forward(q, k, v, beta, s0)
        scan_bf16_backward(q, k, v, beta, saved, inp["d_o"], None)
    e1.record()
    torch.cuda.synchronize(device)
    scan_ms = e0.elapsed_time(e1) / reps
    check_status(device)
    algo = scan_algorithmic_bytes(B, T, H, D)
    pk = peaks()
    hbm_peak = pk.get("hbm_gbs")
    peak_src = "measured" if hbm_peak else "fallback"
    hbm_peak = hbm_peak or 6650.0
    achieved = algo / (scan_ms / 1e3) / 1e9
    traffic = None
    prof = ROOT / "profiles" / "scan_traffic.json"
    if prof.exists():
        try:
            traffic = json.loads(prof.read_text()).get("dram_bytes_per_fwd_bwd")
        except ValueError:
            traffic = None
    roofline = {
        "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
        "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
        "kernel": "delta-scan fwd+bwd (prep, forward, state-gradient, local-gradient kernels)",
        "algorithmic_bytes": algo, "ms": round(scan_ms, 4), "peak_source": peak_src,
    }  # fmt: skip

    # --- end to end through the public API: host buffers in, results out, every step ----------
    # An input pipeline's overlap: step i+1's inputs go in on one stream and step i's results come
    # out on another while the next step computes (two device input sets, two pinned result sets,
    # the copy engines of both directions busy at once). The timed region holds exactly the timed
    # steps' input copies, computation and result copies: it opens as the first one's inputs start
    # in and closes when the last one's results are in host memory.
    names = ("x", "q", "v", "beta", "d_o")
    host = {n: inp[n].cpu().pin_memory() for n in names}
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    sets = [inp, dict(inp, **{n: torch.empty_like(inp[n]) for n in names})]
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    compute = torch.cuda.current_stream(device)
    in_done = [torch.cuda.Event(), torch.cuda.Event()]
    used = [torch.cuda.Event(), torch.cuda.Event()]  # the step that read a set has finished
    outs_host: list = [None, None]
    e2e_steps = max(3, min(args.steps, 20))
    ev0 = torch.cuda.Event(enable_timing=True)

    def copy_in(i: int) -> None:
        with torch.cuda.stream(s_in):
            s_in.wait_event(used[i % 2])
            for n, t in host.items():
                sets[i % 2][n].copy_(t, non_blocking=True)
            in_done[i % 2].record(s_in)

    def pipeline(first: int, count: int):
        copy_in(first)
        for i in range(first, first + count):
            if i + 1 < first + count:
                copy_in(i + 1)
            compute.wait_event(in_done[i % 2])
            st = sets[i % 2]
            lv = [st[n].detach().requires_grad_() for n in ("x", "q", "v", "beta")] + leaves[4:]
            o, grads = step(st, lv)
            results = [o] + [g for g in grads[:4]]
            used[i % 2].record(compute)
            if outs_host[i % 2] is None:
                outs_host[i % 2] = [torch.empty(r.shape, dtype=r.dtype, pin_memory=True) for r in results]
            s_out.wait_stream(compute)
            with torch.cuda.stream(s_out):
                for hst, r in zip(outs_host[i % 2], results, strict=True):
                    r.record_stream(s_out)
                    hst.copy_(r, non_blocking=True)
        return o, grads, results

    pipeline(0, 2)  # warm-up
    compute.wait_stream(s_out)
    torch.cuda.synchronize(device)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    ev0.record(s_in)  # the region opens as the first timed step's inputs start in
    o, grads, results = pipeline(2, e2e_steps)
    compute.wait_stream(s_out)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev1.record(compute)
    torch.cuda.synchronize(device)
    e2e_ms = ev0.elapsed_time(ev1) / e2e_steps
    wall_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    outs_host = outs_host[0]
    d2h = sum(t.numel() * t.element_size() for t in outs_host)
    e2e = {
        "value": round(world * B * T / (e2e_ms / 1e3), 1), "unit": "tokens/s",
        "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 3),
        "host_wall_ms_per_step": round(wall_ms, 3),
    }  # fmt: skip

    # --- the looped model's training step (config 4), data-parallel over the ranks ------------
    del inp, sets, leaves, host, outs_host, results, o, grads, saved
    torch.cuda.empty_cache()
    train = None if args.no_train else train_leg(args, device, world, rank, local)

    # --- CPU baseline: the oracle (float64 C port of the reference path) on rank 0 at N=1 ------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_sample()

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(elapsed_ms / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (config-2 distributions, seeded)",
            "config": {
                "workload": WORKLOAD, "B": B, "T": T, "H": H, "d": D, "width": WIDTH, "chunk": 64,
                "taps": TAPS, "tokens_per_gpu_step": B * T, "l2": "inputs larger than L2 (~1 GB per step), no flush",
                "sharding": "each rank its own (batch x head) units, no collective", "graph": "CUDA graph replay",
            },
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "train_step": train,
            "gpu_launches": launches_per_step * args.steps,
            "gpu_launches_per_step": launches_per_step,
            "clocks": clocks.summary(),
        }  # fmt: skip
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


TRAIN_B, TRAIN_T = 32, 2048  # config 4: rows of 2048 tokens per GPU


def train_leg(args, device, world: int, rank: int, local: int) -> dict:
    """Config 4: the looped d512 model's captured training step, B=32 x T=2048 per GPU, DP over NCCL.

    Forward (13 columns x 8 passes, ACT halting, copy-forward, recomputation), objective, backward,
    the all-reduce of the gradient bucket (N > 1), clip and AdamW: one CUDA graph replay per step.
    Tokens/s = N x B x T / the maximum over ranks of the mean replay time (CUDA events).
    """
    import torch
    import torch.distributed as dist

    from vesper_b200 import _lib
    from vesper_b200.model import Vesper, count_parameters
    from vesper_b200.train import VESPER_S, TrainStep

    cfg = VESPER_S
    model = Vesper(cfg.shape, cfg.vocab, cfg.columns, cfg.t_max, cfg.halt_epsilon,
                   torch.Generator().manual_seed(0)).to(device)  # fmt: skip
    trainer = TrainStep(model, cfg, b=TRAIN_B, n=TRAIN_T, distributed=world > 1, warm=3)
    g = torch.Generator(device=device).manual_seed(99 + rank)
    batches = [torch.randint(0, cfg.vocab, (TRAIN_B, TRAIN_T + 1), device=device, generator=g) for _ in range(2)]
    for i in range(5):  # three eager steps, the capture and two replays
        trainer.load(batches[i % 2][:, :-1], batches[i % 2][:, 1:])
        out = trainer.run()
    torch.cuda.synchronize(device)
    _lib.check_status(device)
    steps = max(1, args.train_steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    e0.record()
    for i in range(steps):
        trainer.load(batches[i % 2][:, :-1], batches[i % 2][:, 1:])
        out = trainer.run()
    e1.record()
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / steps
    if world > 1:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    _lib.check_status(device)
    iters = torch.bincount(out[4].flatten(), minlength=cfg.t_max + 1).tolist()
    loss = float(out[0])
    trainer.release()
    torch.cuda.synchronize(device)
    return {
        "metric": "vesper-s train tokens/s", "value": round(world * TRAIN_B * TRAIN_T / (ms / 1e3), 1),
        "unit": "tokens/s", "n_gpus": world, "ms_per_step": round(ms, 2), "steps": steps, "warmup": 5,
        "scaling": "weak", "dtype": "bf16 autocast (float32 master weights, AdamW)",
        "config": {"workload": "config 4: looped model training step", "params": count_parameters(model),
                   "d_model": cfg.shape.d, "columns": cfg.columns, "t_max": cfg.t_max, "vocab": cfg.vocab,
                   "global_batch": world * TRAIN_B, "seq_len": TRAIN_T, "parallelism": f"dp{world}",
                   "halting": "ACT, random-init head, halt_epsilon 0.01", "recompute": cfg.recompute,
                   "exchange": "one NCCL all-reduce of the float32 gradient bucket, inside the step graph"},
        "pass_counts": iters, "loss": round(loss, 4),
    }  # fmt: skip


def cpu_sample(rows: int = 1) -> dict:
    """The oracle on ``rows`` batch rows of the workload (all heads, all tokens), fwd+bwd."""
    import numpy as np

    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle

    rng = np.random.default_rng(7)
    x = rng.standard_normal((rows, T, WIDTH))
    gain = np.ones(WIDTH)
    taps = 0.5 * rng.standard_normal((TAPS, WIDTH))
    hist = np.zeros((rows, TAPS - 1, WIDTH))
    q = rng.standard_normal((rows, T, H, D))
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    v = rng.standard_normal((rows, T, H, D))
    beta = 1 / (1 + np.exp(-rng.standard_normal((rows, T, H))))
    d_o = rng.standard_normal((rows, T, H, D))
    s0 = np.zeros((rows, H, D, D))
    t0 = time.perf_counter()
    xn, _ = oracle.rms_norm(x, gain)
    k = oracle.keys(xn, hist, taps, H)
    o, _ = oracle.delta_scan(q, k, v, beta, s0)
    dq, dk, dv, dbeta, _ = oracle.delta_scan_grads(q, k, v, beta, s0, d_o, np.zeros_like(s0))
    dz, _, _ = oracle.keys_grads(xn, hist, taps, H, dk)
    oracle.rms_norm_grads(x, gain, dz)
    sec = time.perf_counter() - t0
    return {
        "value": round(rows * T / sec, 1), "unit": "tokens/s", "cores": oracle.threads(),
        "kind": "port", "seconds": round(sec, 3),
        "sample": f"{rows} of {B} batch rows (all {H} heads, T={T}) of config 2, fwd+bwd, float64 C oracle",
        "cpu": _cpu_model(),
    }  # fmt: skip


def _cpu_model() -> str:
    try:
        for ln in Path("/proc/cpuinfo").read_text().splitlines():
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def run_reference(args) -> None:
    """The reference's CPU path (oracle port, all host threads) on rank 0; other ranks exit."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    samples = []
    for _ in range(max(1, args.warmup_ref)):
        cpu_sample(1)
    for _ in range(args.steps_ref or args.steps):
        samples.append(cpu_sample(1))
    secs = sum(s["seconds"] for s in samples)
    tokens = T * len(samples)
    value = tokens / secs
    base = dict(samples[0])
    base["value"] = round(value, 1)
    base["seconds"] = round(secs, 3)
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": len(samples), "warmup": args.warmup, "ms_per_step": round(secs / len(samples) * 1e3, 2),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (config-2 distributions, seeded)", "impl": "reference",
        "config": {"workload": WORKLOAD, "B": B, "T": T, "H": H, "d": D, "width": WIDTH,
                   "sample_per_step": "1 batch row (4096 tokens, 8 heads)"},
        "cpu_baseline": base,
        "e2e": {"value": round(value, 1), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }  # fmt: skip
    print(json.dumps(line), flush=True)


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    p.add_argument("--no-train", action="store_true", help="skip the config-4 training-step leg")
    p.add_argument("--train-steps", type=int, default=5, help="timed training-step replays")
    p.add_argument("--profile-step", action="store_true", help="warm up, run one eager step, exit")
    p.add_argument("--batch", type=int, default=B, help="batch rows per GPU (profiling only; the bench is 8)")
    p.add_argument("--steps-ref", type=int, default=0, help="reference samples (default: min(steps, 10))")
    p.add_argument("--warmup-ref", type=int, default=0)
    args = p.parse_args()
    globals()["B"] = args.batch
    if args.impl == "reference":
        if not args.steps_ref:
            args.steps_ref = min(args.steps, 10)
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
