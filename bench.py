"""Benchmark of the vesper-b200 hot path: config 2 of BASELINE.json on B200s.

One step = the fused key pipeline + RMSNorm + bf16 delta scan, forward and backward, on
B=8, H=8, T=4096, d=128 (width 1024): ``x -> fused_rms_norm -> fused_keys -> delta_scan_fused``
with q, v, the write-strength logits (beta = sigmoid(logits) formed inside the scan's kernels)
and the upstream gradient as further inputs, then the backward through all three (gradients of
x, the gain, the taps, q, v and the logits). Synthetic inputs with the config's
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
    """SM clocks and throttle reasons sampled DURING the timed region.

    NVML is read from a thread every ``period`` seconds (a sample is an instantaneous reading,
    so a timed region of a few milliseconds still gets several); the thread has taken its first
    sample before ``__enter__`` returns. Without NVML it falls back to ``nvidia-smi -lms 100``.
    Reasons recorded: hw_slowdown, hw_thermal_slowdown, sw_thermal_slowdown, sw_power_cap.
    """

    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}  # fmt: skip
    SMI_FIELDS = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu: str, period: float = 0.002) -> None:
        self.gpu, self.period = gpu, period
        self.samples: list[tuple[float, float, set[str]]] = []
        self.proc: subprocess.Popen | None = None
        self.thread = None
        self.source = "none"

    def _nvml_handle(self):
        import pynvml  # nvidia-ml-py

        pynvml.nvmlInit()
        if self.gpu.startswith("GPU-"):
            return pynvml, pynvml.nvmlDeviceGetHandleByUUID(self.gpu)
        return pynvml, pynvml.nvmlDeviceGetHandleByIndex(int(self.gpu))

    def __enter__(self) -> Clocks:
        import threading

        try:
            nv, handle = self._nvml_handle()
            get_reasons = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                nv.nvmlDeviceGetCurrentClocksThrottleReasons
            max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(handle, nv.NVML_CLOCK_SM))
        except Exception:  # noqa: BLE001 - no NVML: the nvidia-smi fallback
            return self._smi_enter()
        self.source = "nvml"
        self.stop = threading.Event()
        first = threading.Event()

        def poll() -> None:
            while True:
                try:
                    mhz = float(nv.nvmlDeviceGetClockInfo(handle, nv.NVML_CLOCK_SM))
                    bits = int(get_reasons(handle))
                    self.samples.append((mhz, max_mhz, {n for n, b in self.REASON_BITS.items() if bits & b}))
                except Exception:  # noqa: BLE001
                    pass
                first.set()
                if self.stop.wait(self.period):
                    return

        self.thread = threading.Thread(target=poll, daemon=True)
        self.thread.start()
        first.wait(5.0)
        self.samples.clear()  # the region opens now
        return self

    def _smi_enter(self) -> Clocks:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )  # fmt: skip
            self.source = "nvidia-smi"
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc: object) -> None:
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            return
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in out.splitlines():
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz, mx = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            self.samples.append((mhz, mx, {n for n, f in zip(names, parts[5:9], strict=True) if f.lower() == "active"}))

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0, "source": self.source}
        reasons: set[str] = set()
        for _, _, r in self.samples:
            reasons |= r
        return {
            "sm_mhz": statistics.median(s[0] for s in self.samples),
            "sm_max_mhz": max(s[1] for s in self.samples),
            "reasons": sorted(reasons),
            "samples": len(self.samples),
            "source": self.source,
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
    # the write-strength logits (beta = sigmoid of them, formed inside the scan's kernels)
    beta = torch.randn(B, T, H, device=device, generator=g).bfloat16()
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
    o, _ = delta_scan_fused(q, k, v, beta, inp["s0"], from_logits=True)
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
    _, _, saved = scan_bf16_forward(q, k, v, beta, s0, True)
    reps = max(5, min(args.steps, 50))
    for _ in range(3):
        scan_bf16_forward(q, k, v, beta, s0, True)
        scan_bf16_backward(q, k, v, beta, saved, inp["d_o"], None, True)
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        _, _, saved = scan_bf16_forward(q, k, v, beta, s0, True)
        scan_bf16_backward(q, k, v, beta, saved, inp["d_o"], None, True)
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
    torch.cuda.empty_cache()
    config3 = None if args.no_config3 else config3_leg(device, world, args.steps)
    torch.cuda.empty_cache()
    config5 = None if args.no_config5 else config5_leg(device, world, rank)
    torch.cuda.empty_cache()
    config1 = config1_leg(device, args.steps) if rank == 0 else None

    # --- CPU baseline: the oracle (float64 C port of the reference path) on rank 0 at N=1 ------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle

        oracle.set_threads(oracle.usable_cores())
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
            "config1": config1, "config3": config3, "config5": config5,
            "gpu_launches": launches_per_step * args.steps,
            "gpu_launches_per_step": launches_per_step,
            "clocks": clocks.summary(),
        }  # fmt: skip
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


C1 = (2, 512, 4, 64)  # config 1: B, T, H, d (fp32 scan)


def scan_f32_algorithmic_bytes(b: int, t: int, h: int, d: int) -> int:
    """HBM bytes of the fp32 scan fwd+bwd: (44d+12) per token-head (float32 I/O) + 5 state passes."""
    return b * t * h * (44 * d + 12) + b * h * 5 * 4 * d * d


def config1_leg(device, steps: int) -> dict:
    """Config 1: ``delta_scan_fused_fp32`` forward+backward at B=2, T=512, H=4, d=64 in float32.

    q, k ~ N(0,1) then L2-normalised per head, v ~ N(0,1), beta = sigmoid(N(0,1)), S0 = 0, the
    loss sum(o * g) with g ~ N(0,1), seed 0. Reports microseconds per forward+backward through the
    public entry point (autograd included) and of the two kernels alone (CUDA events on their
    stream), and the kernels' fraction of the HBM roofline (far from it by nature: 8 sequences,
    each walked token by token).
    """
    import torch
    import torch.nn.functional as F  # noqa: N812

    from vesper_b200.kernels.delta_scan import check_status, delta_scan_fused_fp32, scan_f32_backward, scan_f32_forward

    b, t, h, d = C1
    g = torch.Generator(device=device).manual_seed(0)
    q = F.normalize(torch.randn(b, t, h, d, device=device, generator=g), dim=-1)
    k = F.normalize(torch.randn(b, t, h, d, device=device, generator=g), dim=-1)
    v = torch.randn(b, t, h, d, device=device, generator=g)
    beta = torch.sigmoid(torch.randn(b, t, h, device=device, generator=g))
    s0 = torch.zeros(b, h, d, d, device=device)
    gout = torch.randn(b, t, h, d, device=device, generator=g)
    leaves = [x.detach().requires_grad_() for x in (q, k, v, beta, s0)]

    def api() -> None:
        o, _ = delta_scan_fused_fp32(*leaves)
        torch.autograd.grad([o], leaves, [gout])

    def kernels() -> None:
        _, _, resid = scan_f32_forward(q, k, v, beta, s0, True)
        scan_f32_backward(q, k, v, beta, s0, resid, gout, None)

    reps = max(20, min(steps, 200))
    out = {}
    for name, fn in (("api", api), ("kernels", kernels)):
        for _ in range(5):
            fn()
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn()
        e1.record()
        torch.cuda.synchronize(device)
        out[name] = e0.elapsed_time(e1) / reps * 1e3  # us
    check_status(device)
    algo = scan_f32_algorithmic_bytes(b, t, h, d)
    peak = peaks().get("hbm_gbs") or 6650.0
    achieved = algo / (out["kernels"] / 1e6) / 1e9
    return {
        "metric": "delta-scan fwd+bwd, fp32 (config 1)", "value": round(b * t / (out["api"] / 1e6), 1),
        "unit": "tokens/s", "us_per_fwd_bwd": round(out["api"], 2), "kernel_us_per_fwd_bwd": round(out["kernels"], 2),
        "steps": reps, "dtype": "f32",
        "config": {"workload": "config 1: delta_scan_fused_fp32 fwd+bwd", "B": b, "T": t, "H": h, "d": d},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 5), "traffic": None, "algorithmic_bytes": algo,
                     "kernel": "scan_f32_fwd_kernel + scan_f32_bwd_kernel",
                     "note": "8 sequences walked token by token: latency-bound, not a bandwidth figure"},
    }  # fmt: skip


C3 = {"B": 16, "T": 2048, "d": 512, "heads": 8, "head_dim": 64, "kv_groups": 4, "window": 512, "ffn_mult": 3}


def _kernel_group(name: str) -> str:
    n = name.lower()
    for key, group in (("scan_", "delta-scan"), ("delta_step", "delta-scan"), ("attn_", "attention"),
                       ("nll_", "head loss"), ("keys_", "key filter"),
                       ("rms_", "rmsnorm"), ("column_sum", "rmsnorm"), ("select_rows", "copy-forward/compaction"),
                       ("gather_rows", "copy-forward/compaction"), ("expand_rows", "copy-forward/compaction"),
                       ("compact_", "copy-forward/compaction"), ("gather_slabs", "copy-forward/compaction"),
                       ("flatten_compaction", "copy-forward/compaction"), ("bucket_select", "copy-forward/compaction"), ("relu", "relu^2"), ("rotary", "rotary"),
                       ("gemm", "gemm (cuBLAS)"), ("cutlass", "gemm (cuBLAS)"), ("nvjet", "gemm (cuBLAS)"),
                       ("xmma", "gemm (cuBLAS)"), ("cublas", "gemm (cuBLAS)")):  # fmt: skip
        if key in n:
            return group
    return "torch elementwise/other"


def column_bounds(b: int, t: int) -> dict[str, tuple[str, float]]:
    """Per kernel group of one column fwd+bwd at config 3: (bound, algorithmic bytes or flops)."""
    d, h, dk, w, hidden = C3["d"], C3["heads"], C3["head_dim"], C3["window"], C3["ffn_mult"] * C3["d"]
    hkv = h // C3["kv_groups"]
    tokens = b * t
    linear = 4 * d * d + h * d + d * d + 2 * d * hkv * dk + d * d + 2 * d * hidden  # every weight matrix
    w_eff = sum(min(i + 1, w) for i in range(t))
    attn_fwd = b * h * 4 * dk * w_eff
    return {
        "gemm (cuBLAS)": ("tensor", 6.0 * tokens * linear),
        "attention": ("tensor", 3.5 * attn_fwd),
        "delta-scan": ("hbm", float(scan_algorithmic_bytes(b, t, h, dk))),
        "key filter": ("hbm", float(tokens * (10 * d + 16 * h))),
        # the residual stream is float32: forward reads 4d and writes the bf16 output 2d, backward
        # reads x 4d and dy 2d and writes dx 4d, plus the row statistic both ways; three norms
        "rmsnorm": ("hbm", float(3 * tokens * (16 * d + 8))),
    }


def config3_leg(device, world: int, steps: int) -> dict:
    """Config 3: one column forward+backward in bf16 at d_model 512 (8 x 64 heads, kv_groups 4,
    window 512, relu^2 FFN of 1536), B=16, T=2048 per GPU, weights ~ N(0, 0.02), inputs ~ N(0,1).

    The step (``Column.step`` under bf16 autocast, the loss sum(y * g), gradients of x and every
    parameter) is captured as one CUDA graph and replayed; each rank runs its own 16 rows (batch
    sharding, weak scaling, no collective). Per kernel group: device time from one profiled eager
    step and its algorithmic bound (bytes at the HBM peak or flops at the bf16 tensor peak); the
    column total against the sum of those bounds.
    """
    import torch
    import torch.distributed as dist

    from vesper_b200 import _lib
    from vesper_b200.column import Column, ColumnShape, init_column_state, set_scan

    b, t, d = C3["B"], C3["T"], C3["d"]
    shape = ColumnShape(d=d, heads=C3["heads"], kv_groups=C3["kv_groups"], head_dim=C3["head_dim"],
                        window=C3["window"], rotary_base=10000.0, ffn_mult=C3["ffn_mult"], block=64, key_conv=4)  # fmt: skip
    gen = torch.Generator().manual_seed(3)
    col = Column(shape, gen)
    with torch.no_grad():
        for name, p in col.named_parameters():
            if p.dim() == 2 and "conv_k" not in name:
                p.copy_(0.02 * torch.randn(p.shape, generator=gen))
    col = col.to(device)
    set_scan(col, "fused")
    g = torch.Generator(device=device).manual_seed(5 + int(os.environ.get("RANK", "0")))
    x = torch.randn(b, t, d, device=device, generator=g).requires_grad_()
    up = torch.randn(b, t, d, device=device, generator=g)
    pos = torch.arange(t, device=device).expand(b, t).contiguous()
    params = list(col.parameters())

    def step():
        state = init_column_state(shape, b, 1, torch.bfloat16, device)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y, _, _ = col.step(x, pos, state, 0)
        return torch.autograd.grad([(y.float() * up).sum()], [x, *params])

    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        for _ in range(3):
            step()
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize(device)
    reps = max(3, min(steps, 20))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1) / reps
    if world > 1:
        tt = torch.tensor([ms], device=device)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    _lib.check_status(device)
    del graph
    # per kernel group: one eager step under the profiler (device times of every kernel)
    groups: dict[str, float] = {}
    try:
        from torch.profiler import ProfilerActivity, profile

        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            step()
            torch.cuda.synchronize(device)
        for ev in prof.events():
            if ev.device_type == torch.autograd.DeviceType.CUDA and ev.device_time_total > 0:
                grp = _kernel_group(ev.name)
                groups[grp] = groups.get(grp, 0.0) + ev.device_time_total / 1e3  # ms
    except Exception as exc:  # noqa: BLE001 - the breakdown is optional
        groups = {"error": str(exc)[:200]}
    pk = peaks()
    hbm = pk.get("hbm_gbs") or 6650.0
    tensor = pk.get("bf16_tflops") or 1590.0
    rows = {}
    bound_sum = 0.0
    for grp, (kind, amount) in column_bounds(b, t).items():
        bound_ms = amount / (hbm * 1e9 if kind == "hbm" else tensor * 1e12) * 1e3
        bound_sum += bound_ms
        meas = groups.get(grp)
        rows[grp] = {"bound": kind, "ms": None if meas is None else round(meas, 4), "bound_ms": round(bound_ms, 4),
                     "frac": None if not meas else round(bound_ms / meas, 4)}  # fmt: skip
    for grp, meas in groups.items():
        if grp not in rows and isinstance(meas, float):
            rows[grp] = {"bound": None, "ms": round(meas, 4), "bound_ms": None, "frac": None}
    return {
        "metric": "one column fwd+bwd tokens/s (config 3)", "value": round(world * b * t / (ms / 1e3), 1),
        "unit": "tokens/s", "n_gpus": world, "ms_per_step": round(ms, 4), "steps": reps, "scaling": "weak",
        "dtype": "bf16 autocast", "data": "synthetic (N(0,1) inputs, N(0,0.02) weights)",
        "config": {"workload": "config 3: Column.step fwd+bwd, captured graph", **C3, "parallelism": f"batch x{world}",
                   "ffn": "relu^2 (the reference has no SwiGLU)"},
        "kernels": rows, "bound_sum_ms": round(bound_sum, 4),
        "roofline": {"bound": "mixed", "achieved_ms": round(ms, 4), "bound_ms": round(bound_sum, 4),
                     "frac": round(bound_sum / ms, 4), "peak_hbm_gbs": hbm, "peak_bf16_tflops": tensor,
                     "note": "column time against the sum of its kernel groups' roofline times"},
    }  # fmt: skip


C5 = {"B": 64, "T": 16384, "decode_steps": 256, "chunk": 2048}  # config 5, the whole job's batch


def config5_leg(device, world: int, rank: int) -> dict:
    """Config 5: long-context inference of the config-4 model in bf16, B=64 rows sharded by batch
    over the ranks (64 / N rows each, strong scaling): a T=16384-token prefill (chunked forward,
    2048 tokens a chunk, carried states), then 256 greedy one-token decode steps carrying each
    head's 64 x 64 state, the key histories and the ring windows (one captured graph per step).
    Every token runs all 8 passes (the reference decoder's fixed depth, ``DenseRule``). Token ids
    uniform over [0, 32000). Tokens/s = 64 x (16384 + 256) / the max over ranks of the time.
    """
    import torch
    import torch.distributed as dist

    from vesper_b200 import _lib
    from vesper_b200.decode import BatchedDecoder
    from vesper_b200.model import Vesper
    from vesper_b200.train import VESPER_S

    cfg = VESPER_S
    b = C5["B"] // world
    model = Vesper(cfg.shape, cfg.vocab, cfg.columns, cfg.t_max, cfg.halt_epsilon,
                   torch.Generator().manual_seed(0)).to(device)  # fmt: skip
    from vesper_b200.column import set_scan

    set_scan(model, "fused")
    g = torch.Generator(device=device).manual_seed(500 + rank)
    prompt = torch.randint(0, cfg.vocab, (b, C5["T"]), device=device, generator=g)
    dec = BatchedDecoder(model, cfg.t_max, cfg.vocab, b, torch.bfloat16, warm=2)
    # warm-up on a short prompt: the kernels, the allocator and the step's capture
    dec.prefill(prompt[:, : C5["chunk"]], chunk=C5["chunk"])
    tok = prompt[:, :1]
    for _ in range(4):
        tok, _ = dec.step(tok)
    torch.cuda.synchronize(device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    ev[0].record()
    last = dec.prefill(prompt, chunk=C5["chunk"])
    ev[1].record()
    tok = last.argmax(-1)
    for _ in range(C5["decode_steps"]):
        tok, _ = dec.step(tok)
    ev[2].record()
    torch.cuda.synchronize(device)
    pre_ms, dec_ms = ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2])
    if world > 1:
        t = torch.tensor([pre_ms, dec_ms, pre_ms + dec_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pre_ms, dec_ms, total_ms = (float(x) for x in t.tolist())
    else:
        total_ms = pre_ms + dec_ms
    _lib.check_status(device)
    dec.release()
    steps = C5["decode_steps"]
    total_b = b * world
    return {
        "metric": "long-context inference tokens/s (config 5)",
        "value": round(total_b * (C5["T"] + steps) / (total_ms / 1e3), 1), "unit": "tokens/s", "n_gpus": world,
        "scaling": "strong", "dtype": "bf16 autocast", "data": "synthetic (token ids uniform over [0, 32000))",
        "prefill": {"tokens_per_s": round(total_b * C5["T"] / (pre_ms / 1e3), 1), "ms": round(pre_ms, 2)},
        "decode": {"tokens_per_s": round(total_b * steps / (dec_ms / 1e3), 1), "ms_per_step": round(dec_ms / steps, 4),
                   "steps": steps},
        "config": {"workload": "config 5: prefill T=16384 then 256 greedy decode steps", "B": total_b,
                   "rows_per_gpu": b, "T": C5["T"], "prefill_chunk": C5["chunk"], "passes": cfg.t_max,
                   "exit_rule": "dense (every token all passes, the reference decoder's fixed depth)",
                   "parallelism": f"batch x{world}", "decode_graph": "one captured CUDA graph per step"},
    }  # fmt: skip


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
    beta = 1 / (1 + np.exp(-rng.standard_normal((rows, T, H))))  # write_strength of N(0,1) logits
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
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle

    oracle.set_threads(oracle.usable_cores())  # torchrun exports OMP_NUM_THREADS=1
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


def profile_column(args) -> None:
    """One eager config-3 column forward+backward on ``--batch`` rows after ``--warmup`` warm-ups
    (a single process, for an ncu capture of the attention kernels at a reduced size)."""
    import torch

    from vesper_b200.column import Column, ColumnShape, init_column_state, set_scan

    device = torch.device("cuda", 0)
    b, t, d = args.batch, C3["T"], C3["d"]
    shape = ColumnShape(d=d, heads=C3["heads"], kv_groups=C3["kv_groups"], head_dim=C3["head_dim"],
                        window=C3["window"], rotary_base=10000.0, ffn_mult=C3["ffn_mult"], block=64, key_conv=4)  # fmt: skip
    col = Column(shape, torch.Generator().manual_seed(3)).to(device)
    set_scan(col, "fused")
    g = torch.Generator(device=device).manual_seed(5)
    x = torch.randn(b, t, d, device=device, generator=g).requires_grad_()
    up = torch.randn(b, t, d, device=device, generator=g)
    pos = torch.arange(t, device=device).expand(b, t).contiguous()
    for _ in range(max(args.warmup, 1) + 1):
        state = init_column_state(shape, b, 1, torch.bfloat16, device)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y, _, _ = col.step(x, pos, state, 0)
        torch.autograd.grad([(y.float() * up).sum()], [x, *col.parameters()])
    torch.cuda.synchronize(device)


def profile_copies(args) -> None:
    """The loop's compaction and copy-forward kernels once each, eagerly, on one pass of config 4
    at its measured halting (B=32, T=2048, d=512; 5478 of 65536 tokens active, as after two
    passes), after ``--warmup`` warm-ups: the flat compaction, the bucketed gather of the float32
    residual stream, the expand of the recurrent inputs with carried fallbacks, the key select and
    the attention-output relayout (a single process, for an ncu capture of their DRAM bytes)."""
    import torch

    from vesper_b200.kernels.compact import compact_flat, expand_rows, gather_rows, select_rows
    from vesper_b200.kernels.slabs import SLAB_FIRST

    device = torch.device("cuda", 0)
    b, t, d, h = TRAIN_B, TRAIN_T, 512, 8
    g = torch.Generator(device=device).manual_seed(11)
    active = torch.zeros(b * t, dtype=torch.bool, device=device)
    active[torch.randperm(b * t, device=device, generator=g)[:5478]] = True
    active = active.view(b, t)
    x = torch.randn(1, b * t, d, device=device, generator=g)
    carried = [torch.randn(1, b * t, w, device=device, generator=g).to(torch.bfloat16) for w in (d, d, h)]
    fresh_k = torch.randn(b, t, h, d // h, device=device, generator=g).to(torch.bfloat16)
    carry_k = torch.randn(b, t, h, d // h, device=device, generator=g).to(torch.bfloat16)
    oa = torch.randn(1, b * t, d, device=device, generator=g).to(torch.bfloat16)
    with torch.no_grad():
        for _ in range(max(args.warmup, 1) + 1):
            rows = compact_flat(active, SLAB_FIRST)
            (xc,) = gather_rows(rows, [x])
            comp = [torch.randn(1, b * t, w, device=device, generator=g).to(torch.bfloat16) for w in (d, d, d, h)]
            expand_rows(rows, comp, [None, *carried])
            select_rows(active, [fresh_k], [carry_k])
            assert rows.relayout is not None
            gather_rows(rows.relayout, [oa])
    torch.cuda.synchronize(device)


def breakdown(args) -> None:
    """Device time per kernel of one leg under torch's profiler (CUPTI activity, no ncu):
    ``step`` one config-2 step, ``train`` one config-4 training step (a replay of the captured
    step, as the bench times it), ``decode`` one config-5 decode step (a graph replay) after a
    1024-token prefill. Prints a table by kernel
    group and the top kernels. Times under the profiler are not bench values."""
    import collections

    import torch
    from torch.profiler import ProfilerActivity, profile

    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    if args.breakdown == "step":
        inp = make_inputs(device, 1234)
        leaves = [inp[n].detach().requires_grad_() for n in ("x", "q", "v", "beta", "gain", "taps")]
        for _ in range(3):
            step(inp, leaves)

        def run() -> None:
            step(inp, leaves)
    elif args.breakdown == "train":
        from vesper_b200.model import Vesper
        from vesper_b200.train import VESPER_S, TrainStep

        cfg = VESPER_S
        model = Vesper(cfg.shape, cfg.vocab, cfg.columns, cfg.t_max, cfg.halt_epsilon,
                       torch.Generator().manual_seed(0)).to(device)  # fmt: skip
        model.loop.compact_rows = not args.no_compact
        trainer = TrainStep(model, cfg, b=TRAIN_B, n=TRAIN_T, warm=3)  # captured after 3 eager steps
        g = torch.Generator(device=device).manual_seed(99)
        batch = torch.randint(0, cfg.vocab, (TRAIN_B, TRAIN_T + 1), device=device, generator=g)
        trainer.load(batch[:, :-1], batch[:, 1:])
        for _ in range(5):  # three eager steps, the capture, one replay
            trainer.run()

        def run() -> None:
            trainer.run()
    else:
        from vesper_b200.column import set_scan
        from vesper_b200.decode import BatchedDecoder
        from vesper_b200.model import Vesper
        from vesper_b200.train import VESPER_S

        cfg = VESPER_S
        model = Vesper(cfg.shape, cfg.vocab, cfg.columns, cfg.t_max, cfg.halt_epsilon,
                       torch.Generator().manual_seed(0)).to(device)  # fmt: skip
        set_scan(model, "fused")
        g = torch.Generator(device=device).manual_seed(1)
        prompt = torch.randint(0, cfg.vocab, (C5["B"], 1024), device=device, generator=g)
        dec = BatchedDecoder(model, cfg.t_max, cfg.vocab, C5["B"], torch.bfloat16)
        dec.prefill(prompt, chunk=1024)
        tok = prompt[:, :1]
        for _ in range(4):
            tok, _ = dec.step(tok)
        state = {"tok": tok}

        def run() -> None:
            state["tok"], _ = dec.step(state["tok"])
    torch.cuda.synchronize(device)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        run()
        torch.cuda.synchronize(device)
    groups: dict[str, float] = collections.defaultdict(float)
    kernels: dict[str, list[float]] = collections.defaultdict(lambda: [0.0, 0])
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA and ev.device_time_total > 0:
            groups[_kernel_group(ev.name)] += ev.device_time_total / 1e3
            kernels[ev.name[:70]][0] += ev.device_time_total / 1e3
            kernels[ev.name[:70]][1] += 1
    total = sum(groups.values())
    print(f"{args.breakdown}: device time of the kernels {total:.3f} ms")
    print("| group | ms | share |\n| --- | --- | --- |")
    for name, ms in sorted(groups.items(), key=lambda kv: -kv[1]):
        print(f"| {name} | {ms:.3f} | {100 * ms / total:.1f}% |")
    print("| top kernel | launches | ms |\n| --- | --- | --- |")
    for name, (ms, n) in sorted(kernels.items(), key=lambda kv: -kv[1][0])[:20]:
        print(f"| {name.replace('|', '/')} | {n} | {ms:.3f} |")


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    p.add_argument("--no-train", action="store_true", help="skip the config-4 training-step leg")
    p.add_argument("--no-config3", action="store_true", help="skip the config-3 one-column leg")
    p.add_argument("--no-config5", action="store_true", help="skip the config-5 inference leg")
    p.add_argument("--train-steps", type=int, default=5, help="timed training-step replays")
    p.add_argument("--profile-step", action="store_true", help="warm up, run one eager step, exit")
    p.add_argument("--batch", type=int, default=B, help="batch rows per GPU (profiling only; the bench is 8)")
    p.add_argument("--profile-copies", action="store_true",
                   help="warm up, run the loop's compaction and copy kernels once each on config-4 sizes, exit")
    p.add_argument("--profile-column", action="store_true",
                   help="warm up, run one eager config-3 column fwd+bwd of --batch rows, exit (for ncu)")
    p.add_argument("--no-compact", action="store_true",
                   help="--breakdown train: every pass dense (the loop's compact_rows off), for comparison")
    p.add_argument("--breakdown", choices=("step", "train", "decode"), default=None,
                   help="print one leg's device time per kernel group under torch's profiler, then exit")
    p.add_argument("--steps-ref", type=int, default=0, help="reference samples (default: min(steps, 10))")
    p.add_argument("--warmup-ref", type=int, default=0)
    args = p.parse_args()
    globals()["B"] = args.batch
    if args.breakdown:
        breakdown(args)
        return
    if args.profile_column:
        profile_column(args)
        return
    if args.profile_copies:
        profile_copies(args)
        return
    if args.impl == "reference":
        if not args.steps_ref:
            args.steps_ref = min(args.steps, 10)
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
