#!/usr/bin/env python
"""Benchmark of the WarpForth attention hot path on B200 (libwfattn).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl wfattn|reference]
                    [--workload long_prefill|prefill|prefill_f32|decode|gpt2|gpt2_cached|head_call]

For N > 1 launch one process per GPU:
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P bench.py --gpus N

Workloads (all synthetic, seeded):
  long_prefill (default)  causal prefill [16, 48, 8192, 64] bf16, q/k/v = randn (seed 4);
                          heads split evenly over the N ranks, O all-gathered.
                          One step = the whole batch.  Total work is fixed (strong scaling).
  prefill                 causal prefill [8, 12, 1024, 64] bf16, seed 2 (GPT-2 head shape).
  prefill_f32             the same in f32 (the reference-accurate 3xTF32 tensor-core kernel).
  decode                  one-token decode, B=64, H=25, D=64, bf16 cache padded to 4096,
                          kv_lens ~ U[512, 4096] (seed 3); metric = valid KV bytes / s.
  gpt2                    GPT-2 small random init (seed 1), 32-token prompt, 128 greedy
                          tokens, use_cache=False (the demo's mode), f32.
  gpt2_cached             the same generation with the KV cache (use_cache=True).
  head_call               one GPT-2-small attention call [1, 12, 64, 64] f32, seed 0: latency.

Prints ONE JSON line on rank 0.  `value` is device-timed (CUDA events, inputs
resident in HBM, max over ranks); `e2e` repeats the step through the public
API with the inputs copied from pinned host memory and the result read back
inside the timed region.  The default run (long_prefill) on one GPU also
measures every other workload and reports each under `workloads`, with its own
roofline, clocks, e2e, CPU baseline and, where the reference kernel can run
the case, the reference's compiled kernel timed on the same GPU.

`cpu_baseline` is the demo's torch attention on the host cores
(scaled_dot_product_attention in f32; stock eager GPT-2 for the generation
workloads).  `--impl reference` times the CPU restatement of the reference
kernel (the oracle, f64, all host threads) on a bounded sample of the same
workload; under torchrun only rank 0 runs it.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from dataclasses import dataclass, replace
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_BYTES = 126 * 1024 * 1024


@dataclass(frozen=True)
class Workload:
    name: str
    kind: str  # "prefill", "decode", "gpt2" or "head_call"
    B: int
    H: int
    S: int
    D: int
    seed: int
    dtype: str  # "bf16" or "f32"
    sharded: bool
    description: str
    use_cache: bool = False


WORKLOADS = {
    "long_prefill": Workload("long_prefill", "prefill", 16, 48, 8192, 64, 4, "bf16", True,
                             "head-sharded long-context causal prefill [16,48,8192,64] bf16, "
                             "O all-gathered"),
    "prefill": Workload("prefill", "prefill", 8, 12, 1024, 64, 2, "bf16", False,
                        "causal prefill [8,12,1024,64] bf16 (GPT-2 head shape)"),
    "prefill_f32": Workload("prefill_f32", "prefill", 8, 12, 1024, 64, 2, "f32", False,
                            "causal prefill [8,12,1024,64] f32 (reference-accurate path)"),
    "decode": Workload("decode", "decode", 64, 25, 4096, 64, 3, "bf16", False,
                       "decode q_len=1, B=64 H=25 D=64, bf16 KV cache, kv_lens~U[512,4096]"),
    # S = new tokens per step
    "gpt2": Workload("gpt2", "gpt2", 1, 12, 128, 64, 1, "f32", False,
                     "GPT-2 small random-init (seed 1), 32-token prompt (seed 1), greedy 128 "
                     "new tokens, use_cache=False, every attention through libwfattn (f32)"),
    "gpt2_cached": Workload("gpt2_cached", "gpt2", 1, 12, 128, 64, 1, "f32", False,
                            "GPT-2 small random-init (seed 1), 32-token prompt (seed 1), greedy "
                            "128 new tokens with the KV cache (use_cache=True): prompt through "
                            "the prefill kernel, every new token through the decode kernel",
                            use_cache=True),
    "head_call": Workload("head_call", "head_call", 1, 12, 64, 64, 0, "f32", False,
                          "one GPT-2-small attention call [1,12,64,64] f32, seed 0, causal, "
                          "scale 1/8"),
}
# measured beside the default workload on one GPU, reported under "workloads"
SIDE_WORKLOADS = ("prefill", "prefill_f32", "decode", "gpt2", "gpt2_cached", "head_call")


def prefill_flops(w: Workload, heads: int | None = None) -> int:
    h = w.H if heads is None else heads
    return 4 * w.D * h * w.B * (w.S * (w.S + 1) // 2)


def decode_lens():
    import torch

    return torch.randint(512, 4097, (64,), generator=torch.Generator().manual_seed(3)).to(
        torch.int32)


def load_peaks() -> tuple[dict, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text()), "measured"
        except ValueError:
            pass
    return dict(FALLBACK_PEAKS), "fallback"


def f32_fma_peak(peaks: dict) -> float:
    """CUDA-core f32 FMA peak (TFLOP/s): 148 SMs x 128 lanes x 2 FLOP x max SM clock."""
    return 148 * 128 * 2 * float(peaks.get("sm_max_mhz", 1965.0)) * 1e6 / 1e12


def f32_roof(ctx, D: int) -> dict:
    """Roofline of the f32 prefill path.  head_dim 64 runs on the tensor cores: every product is
    three tf32 MMAs (hi*hi + hi*lo + lo*hi) and tf32 issues at half the bf16 rate, so the ceiling
    for the algorithmic FLOPs is the measured bf16 peak / 6.  Other head dims run on the CUDA
    cores, bounded by the f32 FMA rate."""
    if D == 64:
        return {"bound": "tensor", "peak": float(ctx.peaks["bf16_tflops"]) / 6,
                "peak_source": f"{ctx.peak_src} bf16_tflops / 2 (tf32 rate) / 3 (three tf32 "
                "MMAs per product)", "kernel": "prefill_f32_tc_kernel"}
    return {"bound": "fp32-simt", "peak": f32_fma_peak(ctx.peaks),
            "peak_source": "nominal f32 FMA rate at max SM clock", "kernel": "prefill_f32_kernel"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi during a timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_indices: list[int]) -> None:
        self.indices = gpu_indices
        self.proc = None
        self.t0 = 0.0

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", ",".join(map(str, self.indices))],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        self.t0 = time.time()

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        # make sure at least a couple of samples were taken
        while time.time() - self.t0 < 0.5:
            time.sleep(0.05)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons, n = [], [], set(), 0
        for line in out.splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            n += 1
            for name, val in zip(self.REASONS, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": sorted(reasons),
                "samples": n}


def physical_gpu_indices(n: int) -> list[int]:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [int(x) for x in vis.split(",") if x.strip().isdigit()]
        if len(ids) >= n:
            return ids[:n]
    return list(range(n))


def host_threads() -> int:
    """Host cores this process may run on.  torchrun sets OMP_NUM_THREADS=1 for every rank, so
    the CPU legs pass their thread count explicitly instead of taking OpenMP's default."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ------------------------------------------------------------------ CPU: the oracle (reference arm)
def oracle_sample(w: Workload, target_s: float, threads: int) -> dict:
    """Times the oracle (f64 restatement of the reference kernel) on a bounded sample.

    Prefill: the last R query rows of `nh` heads of the workload's shape (the
    costliest rows: each sees all S keys).  Decode: `nb` whole sequences.
    Returns value in the workload's metric unit plus a description.
    """
    import numpy as np
    import torch

    import oracle

    if w.kind == "gpt2":
        return gpt2_cpu_sample(w, target_s, threads)
    g = torch.Generator().manual_seed(w.seed)

    def bf(t):
        return t.to(torch.bfloat16).float().numpy() if w.dtype == "bf16" else t.numpy()

    if w.kind == "head_call":
        q, k, v = (torch.randn(w.B, w.H, w.S, w.D, generator=g).numpy() for _ in range(3))
        n, dt = 0, 0.0
        t0 = time.perf_counter()
        while dt < 0.5 * target_s:
            oracle.attention(q, k, v, nthreads=threads)
            n += 1
            dt = time.perf_counter() - t0
        return {"value": dt / n * 1e6, "unit": "us per call", "seconds": dt,
                "sample": f"oracle (f64) on the whole [1,12,64,64] call, {n} calls"}
    if w.kind == "prefill":
        def run(nh, rows):
            q, k, v = (bf(torch.randn(1, nh, w.S, w.D, generator=g)) for _ in range(3))
            t0 = time.perf_counter()
            oracle.attention(q, k, v, row_range=(w.S - rows, w.S), nthreads=threads)
            dt = time.perf_counter() - t0
            pairs = nh * sum(i + 1 for i in range(w.S - rows, w.S))
            return dt, 4 * w.D * pairs

        rows_total = 64
        while True:
            nh = max(1, math.ceil(rows_total / w.S))
            rows = max(1, min(w.S, rows_total // nh))
            dt, fl = run(nh, rows)
            if dt >= 0.5 * target_s or nh >= 4 * w.H:
                break
            rows_total = int(rows_total * min(16.0, max(1.5, target_s / max(dt, 1e-3))))
        return {"value": fl / dt / 1e12, "unit": "TFLOP/s", "seconds": dt,
                "sample": f"oracle (f64) on the last {rows} query rows of {nh} head(s) "
                          f"of shape S={w.S}, D={w.D}: {fl:.3e} FLOP in {dt:.2f} s"}
    # decode: whole sequences of the workload (all heads), repeated to reach the target time
    lens = decode_lens().numpy()
    nb, reps = 4, 1
    while True:
        sel = lens[:nb]
        q = bf(torch.randn(nb, w.H, 1, w.D, generator=g))
        lm = int(sel.max())
        k, v = (bf(torch.randn(nb, w.H, lm, w.D, generator=g)) for _ in range(2))
        t0 = time.perf_counter()
        for _ in range(reps):
            oracle.attention(q, k, v, causal=False, kv_lens=sel.astype(np.int32),
                             nthreads=threads)
        dt = time.perf_counter() - t0
        by = reps * int(sel.sum()) * w.H * w.D * 2 * 2
        if dt >= 0.5 * target_s:
            break
        grow = min(16.0, max(1.5, target_s / max(dt, 1e-3)))
        if nb < w.B:
            nb = min(w.B, int(math.ceil(nb * grow)))
        else:
            reps = int(math.ceil(reps * grow))
    return {"value": by / dt / 1e9, "unit": "GB/s", "seconds": dt,
            "sample": f"oracle (f64) on {nb} whole sequence(s) x {w.H} heads, {reps} pass(es): "
                      f"{by} valid KV bytes (bf16-equivalent) in {dt:.2f} s"}


# ------------------------------------------------------------------ CPU: the demo's torch attention
def torch_cpu_sample(w: Workload, target_s: float, threads: int) -> dict:
    """The demo's torch attention on the host cores: scaled_dot_product_attention in f32 (the
    golden path of the GPT-2 head call), grown until it takes about `target_s`; stock eager
    GPT-2 for the generation workloads."""
    import torch
    import torch.nn.functional as F

    if w.kind == "gpt2":
        return gpt2_cpu_sample(w, target_s, threads)
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(w.seed)
    if w.kind == "head_call":
        q, k, v = (torch.randn(w.B, w.H, w.S, w.D, generator=g) for _ in range(3))
        for _ in range(3):
            F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=w.D ** -0.5)
        n, dt = 0, 0.0
        t0 = time.perf_counter()
        while dt < 0.5 * target_s:
            F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=w.D ** -0.5)
            n += 1
            dt = time.perf_counter() - t0
        return {"value": dt / n * 1e6, "unit": "us per call", "seconds": dt,
                "sample": f"torch SDPA f32 on the whole call, {n} calls, {threads} threads"}
    if w.kind == "prefill":
        nh = 1
        while True:
            q, k, v = (torch.randn(1, nh, w.S, w.D, generator=g) for _ in range(3))
            F.scaled_dot_product_attention(q[:, :1], k[:, :1], v[:, :1], is_causal=True)
            t0 = time.perf_counter()
            F.scaled_dot_product_attention(q, k, v, is_causal=True, scale=w.D ** -0.5)
            dt = time.perf_counter() - t0
            if dt >= 0.5 * target_s or nh >= w.B * w.H:
                break
            nh = min(w.B * w.H, max(nh + 1, int(nh * min(8.0, target_s / max(dt, 1e-3)))))
        fl = 4 * w.D * nh * (w.S * (w.S + 1) // 2)
        return {"value": fl / dt / 1e12, "unit": "TFLOP/s", "seconds": dt,
                "sample": f"torch SDPA f32 (causal) on {nh} head(s) of S={w.S}, D={w.D}: "
                          f"{fl:.3e} FLOP in {dt:.2f} s, {threads} threads"}
    # decode: torch SDPA per sequence over its valid keys (ragged), f32
    lens = decode_lens()
    q = torch.randn(w.B, w.H, 1, w.D, generator=g)
    nb, reps = 8, 1
    kv = [(torch.randn(1, w.H, int(lens[b]), w.D, generator=g),
           torch.randn(1, w.H, int(lens[b]), w.D, generator=g)) for b in range(w.B)]
    while True:
        t0 = time.perf_counter()
        for _ in range(reps):
            for b in range(nb):
                F.scaled_dot_product_attention(q[b:b + 1], kv[b][0], kv[b][1])
        dt = time.perf_counter() - t0
        by = reps * int(lens[:nb].sum()) * w.H * w.D * 2 * 2
        if dt >= 0.5 * target_s:
            break
        grow = min(16.0, max(1.5, target_s / max(dt, 1e-3)))
        if nb < w.B:
            nb = min(w.B, int(math.ceil(nb * grow)))
        else:
            reps = int(math.ceil(reps * grow))
    return {"value": by / dt / 1e9, "unit": "GB/s", "seconds": dt,
            "sample": f"torch SDPA f32 per sequence on {nb} sequence(s) x {w.H} heads, {reps} "
                      f"pass(es): {by} valid KV bytes (bf16-equivalent) in {dt:.2f} s, "
                      f"{threads} threads"}


def gpt2_cpu_sample(w: Workload, target_s: float, threads: int) -> dict:
    """Stock eager GPT-2 on the host cores (the demo's torch attention), greedy tokens/s."""
    import torch

    from warpforth_b200 import gpt2

    torch.set_num_threads(threads)
    model = gpt2.random_gpt2(seed=1, device="cpu")
    prompt = gpt2.synthetic_prompt(32, seed=1)
    n = 4
    while True:
        t0 = time.perf_counter()
        gpt2.generate(model, prompt, n, use_cache=w.use_cache)
        dt = time.perf_counter() - t0
        if dt >= 0.5 * target_s or n >= 128:
            break
        n = min(128, max(n + 1, int(n * min(8.0, target_s / max(dt, 1e-3)))))
    return {"value": n / dt, "unit": "tokens/s", "seconds": dt,
            "sample": f"stock eager GPT-2 (torch CPU, {threads} threads, use_cache="
                      f"{w.use_cache}): the first {n} greedy tokens of the same prompt in "
                      f"{dt:.2f} s"}


def cpu_baseline_of(w: Workload, target_s: float) -> dict:
    threads = host_threads()
    r = torch_cpu_sample(w, target_s, threads)
    return {"value": r["value"], "unit": r["unit"], "cores": threads, "kind": "reference",
            "what": "the demo's torch attention on the host cores (torch "
                    "scaled_dot_product_attention f32; stock eager GPT-2 for generation)",
            "sample": r["sample"]}


def run_reference(args, w: Workload) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = host_threads()
    metric, unit, hib = metric_of(w)
    vals = []
    sample = None
    for i in range(args.warmup + args.steps):
        r = oracle_sample(w, args.ref_step_seconds, threads)
        sample = r["sample"]
        if i >= args.warmup:
            vals.append(r["value"])
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": hib, "dtype": "f32" if w.kind == "gpt2" else "f64",
        "data": "synthetic", "config": config_of(w, args.gpus),
        "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "vs_baseline": None,
    }
    print(json.dumps(line), flush=True)


def metric_of(w: Workload) -> tuple[str, str, bool]:
    if w.kind == "decode":
        return "decode attention KV GB/s per B200", "GB/s", True
    if w.kind == "gpt2":
        return "GPT-2 gen tokens/s", "tokens/s", True
    if w.kind == "head_call":
        return "GPT-2 attention call latency", "us per call", False
    return "causal SDPA TFLOP/s", "TFLOP/s", True


def config_of(w: Workload, n: int) -> dict:
    cfg = {"workload": w.description, "batch": w.B, "heads": w.H, "head_dim": w.D,
           "seed": w.seed}
    if w.kind == "gpt2":
        cfg.update({"model": "gpt2-small (12 layers, d_model 768, vocab 50257, ctx 1024)",
                    "prompt_len": 32, "new_tokens": w.S, "use_cache": w.use_cache,
                    "parallelism": f"replicas/{n}" if n > 1 else "single",
                    "l2": "not applicable (end-to-end generation)"})
        return cfg
    if w.kind == "head_call":
        cfg.update({"seq_len": w.S, "causal": True, "parallelism": "single",
                    "l2": "inputs resident in L2 (0.6 MB; a latency measurement)"})
        return cfg
    if w.kind == "prefill":
        cfg.update({"seq_len": w.S, "causal": True,
                    "parallelism": f"heads/{n}" if w.sharded and n > 1 else
                    (f"replicas/{n}" if n > 1 else "single"),
                    "l2": "inputs larger than L2 (126 MB)" if w.S >= 4096 else
                    "L2 flushed between timed steps (a 256 MB read)"})
    else:
        cfg.update({"max_kv_len": w.S, "kv_lens": "U[512,4096] seed 3 (sum 142652)",
                    "parallelism": f"replicas/{n}" if n > 1 else "single",
                    "l2": "inputs larger than L2 (913 MB of K/V read per step, 126 MB L2)"})
    return cfg


# ------------------------------------------------------------------ GPU side
class Ctx:
    """Process-group plumbing shared by the GPU legs."""

    def __init__(self) -> None:
        import torch
        import torch.distributed as dist

        self.torch, self.dist = torch, dist
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local_rank)
        self.dev = torch.device("cuda", self.local_rank)
        if self.world > 1:
            from datetime import timedelta

            dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=self.dev)
        self.stream = torch.cuda.current_stream(self.dev)
        self.peaks, self.peak_src = load_peaks()
        self._flush = None

    def barrier(self) -> None:
        if self.world > 1:
            self.dist.barrier()

    def max_over_ranks(self, x: float) -> float:
        if self.world == 1:
            return x
        t = self.torch.tensor([x], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def min_over_ranks(self, x: float) -> float:
        return -self.max_over_ranks(-x)

    def flush_l2(self) -> None:
        """Evicts L2 by reading a 256 MB buffer (twice L2): clean lines, no write-back for
        the next kernel to pay."""
        if self._flush is None:
            self._flush = self.torch.ones(2 * L2_BYTES // 4, dtype=self.torch.float32,
                                          device=self.dev)
        self._flush.sum()

    def clocks(self):
        return ClockSampler(physical_gpu_indices(self.world)) if self.rank == 0 else None

    def event(self):
        return self.torch.cuda.Event(enable_timing=True)

    def close(self) -> None:
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


def time_steps(ctx: Ctx, fn, steps: int, flush: bool) -> tuple[float, list[float], dict | None]:
    """Times `steps` calls of fn with CUDA events on the current stream; returns the total ms
    (the sum of per-step times when L2 is flushed between steps), the per-step times and the
    clocks seen.  Bracketed by a barrier and a synchronize on both sides."""
    torch = ctx.torch
    torch.cuda.synchronize()
    ctx.barrier()
    clocks = ctx.clocks()
    if clocks:
        clocks.start()
    ev = [(ctx.event(), ctx.event()) for _ in range(steps)]
    t0, t1 = ctx.event(), ctx.event()
    torch.cuda.synchronize()
    ctx.barrier()
    t0.record(ctx.stream)
    for i in range(steps):
        if flush:
            ctx.flush_l2()
        ev[i][0].record(ctx.stream)
        fn()
        ev[i][1].record(ctx.stream)
    t1.record(ctx.stream)
    torch.cuda.synchronize()
    ctx.barrier()
    info = clocks.stop() if clocks else None
    per = [a.elapsed_time(b) for a, b in ev]
    total = sum(per) if flush else t0.elapsed_time(t1)
    return total, per, info


def graph_of(ctx: Ctx, fn):
    """fn captured once in a CUDA graph: the device timing then holds the GPU work of the
    library call, not the Python/ctypes launch path (`e2e` goes through that path)."""
    torch = ctx.torch
    fn()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g


def timed_e2e(ctx: Ctx, one, steps: int, warmup: int, flush: bool) -> float:
    """Mean ms of `one` (copies in, compute, copy out) over `steps`, max over ranks."""
    torch = ctx.torch
    for _ in range(warmup):
        one()
    torch.cuda.synchronize()
    ctx.barrier()
    a, b = ctx.event(), ctx.event()
    tot = 0.0
    for _ in range(steps):
        if flush:
            ctx.flush_l2()
        torch.cuda.synchronize()
        a.record(ctx.stream)
        one()
        b.record(ctx.stream)
        torch.cuda.synchronize()
        tot += a.elapsed_time(b)
    ctx.barrier()
    return ctx.max_over_ranks(tot / steps)


def run_prefill(args, ctx: Ctx, w: Workload) -> dict:
    torch = ctx.torch
    from warpforth_b200 import warpforth as wf
    from warpforth_b200.sharded import ShardedPrefill

    world, dev = ctx.world, ctx.dev
    tdt = torch.bfloat16 if w.dtype == "bf16" else torch.float32
    flush = w.S < 4096  # the [8,12,1024] inputs (50-100 MB) fit in L2; 1.6 GB do not
    torch.manual_seed(w.seed)
    sp = None
    parity = None
    if w.sharded:
        q, k, v = (torch.randn(w.B, w.H, w.S, w.D, device=dev, dtype=tdt) for _ in range(3))
        sp = ShardedPrefill(w.B, w.H, w.S, w.D, dtype=tdt, device=dev,
                            chunks=args.chunks or None, transport=args.transport)
        qs, ks, vs = sp.shard(q), sp.shard(k), sp.shard(v)
        units = prefill_flops(w)  # whole job per step
        kernel_flops = prefill_flops(w, sp.local_heads)

        def step():
            # this rank's heads; the gather of O rides along (peer stores from the
            # kernel, or per-chunk NCCL all-gathers overlapping compute)
            sp(qs, ks, vs)

        timed = step
    else:
        q, k, v = (torch.randn(w.B, w.H, w.S, w.D, device=dev).to(tdt) for _ in range(3))
        out = torch.empty_like(q)
        units = prefill_flops(w) * world  # every rank runs one replica
        kernel_flops = prefill_flops(w)

        def step():
            wf.attention(q, k, v, out=out)

        timed = None
    for _ in range(args.warmup):
        if flush:
            ctx.flush_l2()
        step()
    if timed is None:
        timed = graph_of(ctx, step).replay
    total_ms, per, clock_info = time_steps(ctx, timed, args.steps, flush)
    kernel_ms = statistics.mean(per)
    if w.sharded:
        # every rank recomputes the whole output on its own GPU with the same kernel and
        # compares it bit for bit with the gathered one (all steps had these inputs)
        got = sp.output_view()
        ref = torch.empty((w.B, w.H, w.S, w.D), dtype=tdt, device=dev)
        wf.attention_gather(q, k, v, [ref])
        torch.cuda.synchronize()
        exact = float(torch.equal(got, ref))
        rel = float((got.float() - ref.float()).abs().max() / ref.float().abs().max())
        parity = {"heads_checked": w.B * w.H, "bit_exact": ctx.min_over_ranks(exact) == 1.0,
                  "max_rel_err": ctx.max_over_ranks(rel), "ranks_checked": world,
                  "reference": "every rank: the same kernel for all heads on its own GPU"}
        del ref, got
        # the roofline's kernel time: this rank's heads alone, without the final barrier
        ev = [(ctx.event(), ctx.event()) for _ in range(args.steps)]
        for a, b in ev:
            a.record(ctx.stream)
            sp.compute_local(qs, ks, vs)
            b.record(ctx.stream)
        torch.cuda.synchronize()
        kernel_ms = statistics.mean(a.elapsed_time(b) for a, b in ev)
        ctx.barrier()
        # the same heads computed into a local buffer, with no gather at all: what the
        # rank's kernel would take if nothing had to cross NVLink
        local_out = torch.empty((w.B, sp.local_heads, w.S, w.D), dtype=tdt, device=dev)
        outs = sp.split_local(local_out)
        ev = [(ctx.event(), ctx.event()) for _ in range(args.steps)]
        for a, b in ev:
            a.record(ctx.stream)
            for c in range(sp.chunks):
                wf.attention(qs[c], ks[c], vs[c], out=outs[c])
            b.record(ctx.stream)
        torch.cuda.synchronize()
        compute_ms = ctx.max_over_ranks(statistics.mean(a.elapsed_time(b) for a, b in ev))
        del local_out, outs
        ctx.barrier()
    total_ms = ctx.max_over_ranks(total_ms)
    kernel_ms = ctx.max_over_ranks(kernel_ms)
    ms_per_step = total_ms / args.steps
    value = units / (ms_per_step / 1e3) / 1e12

    # ---------------- end to end through the public API with host buffers
    steps = max(1, min(args.steps, args.e2e_steps))
    g = torch.Generator().manual_seed(w.seed + 1000)
    heads = sp.local_heads if sp is not None else w.H
    shape = (w.B, heads, w.S, w.D)
    host = [torch.randn(*shape, generator=g).to(tdt).pin_memory() for _ in range(3)]
    dev_in = [torch.empty(shape, dtype=tdt, device=dev) for _ in range(3)]
    # One GPU holds every head: the step goes through wf.attention in batch chunks, so the
    # copies in (one stream) and out (another stream) overlap other chunks' compute.
    # Several GPUs: this rank's heads go in, the gathered output comes out on rank 0.
    pipelined = w.B >= 4 and (sp is None or ctx.world == 1)
    if sp is not None and not pipelined:
        host_out = torch.empty((w.B, w.H, w.S, w.D), dtype=tdt).pin_memory() \
            if ctx.rank == 0 else None
    else:
        res = torch.empty(shape, dtype=tdt, device=dev)
        host_out = torch.empty(shape, dtype=tdt).pin_memory()
    cs_in, cs_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    nchunk = 4
    bounds = [(c * w.B // nchunk, (c + 1) * w.B // nchunk) for c in range(nchunk)]

    def one():
        if pipelined:
            main = torch.cuda.current_stream(dev)
            cs_in.wait_stream(main)
            cs_out.wait_stream(main)
            arrived = []
            with torch.cuda.stream(cs_in):
                for b0, b1 in bounds:
                    for h_, d_ in zip(host, dev_in):
                        d_[b0:b1].copy_(h_[b0:b1], non_blocking=True)
                    e = torch.cuda.Event()
                    e.record(cs_in)
                    arrived.append(e)
            for (b0, b1), e in zip(bounds, arrived):
                main.wait_event(e)
                wf.attention(*(t[b0:b1] for t in dev_in), out=res[b0:b1])
                done = torch.cuda.Event()
                done.record(main)
                cs_out.wait_event(done)
                with torch.cuda.stream(cs_out):
                    host_out[b0:b1].copy_(res[b0:b1], non_blocking=True)
            main.wait_stream(cs_out)
            return
        for h_, d_ in zip(host, dev_in):
            d_.copy_(h_, non_blocking=True)
        out_ = sp(*(sp.split_local(t) for t in dev_in))
        if host_out is not None:
            host_out.copy_(out_, non_blocking=True)

    e2e_ms = timed_e2e(ctx, one, steps, args.warmup, flush)
    e2e = {"value": units / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
           "steps": steps, "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host),
           "d2h_bytes_per_step": host_out.numel() * host_out.element_size() if host_out is not None
           else 0,
           "path": ("warpforth_b200.warpforth.attention (ctypes) -> libwfattn C ABI, pinned host "
                    f"buffers; the batch in {nchunk} chunks, copies in and out on two side "
                    "streams overlapping the other chunks' compute") if pipelined else
                   "ShardedPrefill -> libwfattn C ABI, this rank's q/k/v in from pinned host "
                   "buffers, the gathered output out on rank 0"}
    del host, dev_in

    if w.dtype == "f32":
        roof = f32_roof(ctx, w.D)
    else:
        key = "bf16_tflops_sustained" if (w.sharded and ms_per_step > 1000) else "bf16_tflops"
        roof = {"bound": "tensor", "peak": float(ctx.peaks[key]),
                "peak_source": f"{ctx.peak_src} {key}",
                "kernel": "prefill_bf16_2q_kernel" if (w.S + 255) // 256 * w.B * heads >= 148
                else "prefill_bf16_kernel"}
    achieved = kernel_flops / (kernel_ms / 1e3) / 1e12
    traffic = load_traffic(w)
    if traffic is not None and w.sharded:
        traffic = int(traffic * heads / w.H)  # this rank's launch
    roof.update({"achieved": achieved, "unit": "TFLOP/s", "frac": achieved / roof["peak"],
                 "kernel_ms": kernel_ms, "traffic": traffic, "traffic_source": TRAFFIC_SOURCE,
                 "algorithmic_flop_per_launch": kernel_flops})
    line = {
        "metric": "causal SDPA TFLOP/s", "value": value, "unit": "TFLOP/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "strong" if w.sharded else "weak",
        "vs_baseline": None, "dtype": w.dtype, "data": "synthetic",
        "config": dict(config_of(w, world), **({"gather": sp.transport} if sp else {}),
                       device_timing="per-rank CUDA events around each step, max over ranks"
                       if w.sharded else "CUDA events around each step's library call, "
                       "replayed from a CUDA graph"),
        "roofline": roof, "e2e": e2e,
        # kernels of this library per timed step, all ranks: one launch per head chunk
        "gpu_launches": args.steps * world * (sp.chunks if sp is not None else 1),
        "clocks": clock_info,
    }
    if parity is not None:
        line["parity"] = parity
    if sp is not None and world > 1:
        # NVLink volume of the gather per rank and step; the fused kernel can finish no
        # sooner than the slower of its compute alone and its link time at the measured
        # 770 GB/s per direction of a peer copy
        share = w.B * sp.local_heads * w.S * w.D * (2 if tdt == torch.bfloat16 else 4)
        others = share * (world - 1)
        link_ms = others / 770e9 * 1e3
        line["gather"] = {
            "transport": sp.transport,
            "bytes_in_per_rank": others, "bytes_out_per_rank":
                share if sp.transport == "multicast" else others,
            "compute_only_ms": compute_ms, "fused_kernel_ms": kernel_ms,
            "link_bound_ms": link_ms, "link_gbs": 770.0,
            "fused_frac": max(compute_ms, link_ms) / kernel_ms,
            "what": "bytes_in: the other ranks' shares of O; bytes_out: this rank's share, once "
                    "(multicast: the NVLink switch replicates it, its own copy included) or once "
                    "per other rank; compute_only: this rank's heads into a local buffer; "
                    "fused_frac = max(compute_only, link_bound) / fused kernel"}
    if not w.sharded and w.dtype == "f32" and ctx.rank == 0:
        line["reference_ptx"] = ref_ptx_prefill(ctx, w, q, k, v, out, args)
    if sp is not None:
        sp.close()  # collective: unmaps and frees the peer output buffers
    return line


def run_decode(args, ctx: Ctx, w: Workload) -> dict:
    torch = ctx.torch
    from warpforth_b200 import warpforth as wf

    dev, world = ctx.dev, ctx.world
    tdt = torch.bfloat16
    torch.manual_seed(w.seed)
    lens = decode_lens().to(dev)
    kc = torch.randn(w.B, w.H, w.S, w.D, device=dev, dtype=tdt)
    vc = torch.randn(w.B, w.H, w.S, w.D, device=dev, dtype=tdt)
    qd = torch.randn(w.B, w.H, w.D, device=dev, dtype=tdt)
    od = torch.empty(w.B, w.H, w.D, device=dev, dtype=torch.float32)
    ws = wf.DecodeWorkspace()
    kv_bytes = int(decode_lens().sum()) * w.H * w.D * 2 * 2

    def step():
        wf.decode(qd, kc, vc, lens, out=od, workspace=ws)

    for _ in range(args.warmup):
        step()
    # the 913 MB of K/V read per step exceed L2: no flush
    total_ms, per, clock_info = time_steps(ctx, graph_of(ctx, step).replay, args.steps, False)
    total_ms = ctx.max_over_ranks(total_ms)
    # the roofline's kernel: the split kernel alone (the combine kernel reads 26 MB)
    split_ms = ctx.max_over_ranks(statistics.mean(per))
    ms_per_step = total_ms / args.steps
    value = kv_bytes * world / (ms_per_step / 1e3) / 1e9

    # end to end, decode serving: the KV cache is resident state; a step's inputs are the new
    # query token, the new K/V row of every (batch, head) and the lengths
    g = torch.Generator().manual_seed(w.seed + 1000)
    # One pinned staging buffer per step, sent in one copy: the new query, K and V rows
    # (bf16 [3, B, H, D]), the rows' cache positions (int64 [B], lens - 1, known on the host)
    # and the lengths (int32 [B]).
    n_rows = 3 * w.B * w.H * w.D
    row_bytes, pos_bytes = n_rows * 2, w.B * 8
    stage_h = torch.empty(row_bytes + pos_bytes + w.B * 4, dtype=torch.uint8).pin_memory()
    stage_h[:row_bytes].view(tdt).copy_(torch.randn(n_rows, generator=g).to(tdt))
    lens_cpu = decode_lens()
    stage_h[row_bytes:row_bytes + pos_bytes].view(torch.int64).copy_(lens_cpu.long() - 1)
    stage_h[row_bytes + pos_bytes:].view(torch.int32).copy_(lens_cpu)
    stage_d = torch.empty_like(stage_h, device=dev)
    rows = stage_d[:row_bytes].view(tdt).view(3, w.B, w.H, w.D)
    qn, knew, vnew = rows[0], rows[1], rows[2]
    pos = stage_d[row_bytes:row_bytes + pos_bytes].view(torch.int64)
    lens_d = stage_d[row_bytes + pos_bytes:].view(torch.int32)
    out_h = torch.empty((w.B, w.H, w.D), dtype=torch.float32).pin_memory()
    bidx = torch.arange(w.B, device=dev)

    def one():
        stage_d.copy_(stage_h, non_blocking=True)
        kc[bidx, :, pos] = knew
        vc[bidx, :, pos] = vnew
        wf.decode(qn, kc, vc, lens_d, out=od, workspace=ws)
        out_h.copy_(od, non_blocking=True)

    steps = max(1, min(args.steps, args.e2e_steps))
    e2e_ms = timed_e2e(ctx, one, steps, args.warmup, False)
    e2e = {"value": kv_bytes * world / (e2e_ms / 1e3) / 1e9, "unit": "GB/s",
           "ms_per_step": e2e_ms, "steps": steps,
           "h2d_bytes_per_step": stage_h.numel(),
           "d2h_bytes_per_step": out_h.numel() * 4,
           "path": "warpforth_b200.warpforth.decode (ctypes) -> libwfattn C ABI; the step's "
                   "new q/K/V rows, cache positions and lengths in one pinned copy, the K/V rows "
                   "scattered into the resident cache"}
    peak = float(ctx.peaks["hbm_gbs"])
    achieved = kv_bytes / (split_ms / 1e3) / 1e9
    roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
            "frac": achieved / peak, "peak_source": f"{ctx.peak_src} hbm_gbs",
            "kernel": "decode_split_kernel + decode_combine_kernel (one library call)",
            "kernel_ms": split_ms, "traffic": load_traffic(w), "traffic_source": TRAFFIC_SOURCE,
            "algorithmic_bytes_per_launch": kv_bytes}
    return {
        "metric": "decode attention KV GB/s per B200", "value": value, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": dict(config_of(w, world), device_timing="CUDA events "
                                            "around each step's library call, replayed from a "
                                            "CUDA graph"),
        "roofline": roof, "e2e": e2e, "gpu_launches": args.steps * world * 2,
        "clocks": clock_info,
    }


def run_head_call(args, ctx: Ctx, w: Workload) -> dict:
    """Config 1: one [1,12,64,64] f32 attention call; latency per call."""
    torch = ctx.torch
    from warpforth_b200 import warpforth as wf

    dev = ctx.dev
    torch.manual_seed(w.seed)
    q, k, v = (torch.randn(w.B, w.H, w.S, w.D).to(dev) for _ in range(3))
    out = torch.empty_like(q)

    def step():
        wf.attention(q, k, v, out=out)

    for _ in range(args.warmup):
        step()
    n_calls = 100  # a step of ~10 us is timed as the mean of 100 graph-replayed calls
    g = graph_of(ctx, step)
    total_ms, per, clock_info = time_steps(ctx, lambda: [g.replay() for _ in range(n_calls)],
                                           args.steps, False)
    us = total_ms / args.steps / n_calls * 1e3
    # end to end: copies in, the call through the reference-shaped ABI (12 launches of one
    # head each, as demo/gpt2_generate.py:42-50 does), copy out
    # q, k, v staged in one pinned buffer and sent in one copy
    host_qkv = torch.stack([t.cpu() for t in (q, k, v)]).pin_memory()
    host = [host_qkv[0], host_qkv[1], host_qkv[2]]
    host_out = torch.empty_like(host[0]).pin_memory()
    kern = wf.AttentionKernel()
    dqkv = torch.empty_like(host_qkv, device=dev)
    dq, dk, dv = dqkv[0], dqkv[1], dqkv[2]

    def one():
        dqkv.copy_(host_qkv, non_blocking=True)
        for h in range(w.H):
            kern(dq[0, h], dk[0, h], dv[0, h], out[0, h], w.S, w.D)
        host_out.copy_(out, non_blocking=True)

    e2e_ms = timed_e2e(ctx, one, 20, args.warmup, False)
    flops = prefill_flops(w)
    roof = f32_roof(ctx, w.D)
    achieved = flops / (us / 1e6) / 1e12
    line = {
        "metric": "GPT-2 attention call latency", "value": us, "unit": "us per call",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(config_of(w, 1), device_timing=f"CUDA events around {n_calls} graph "
                       "replays of the batched library call per step"),
        "roofline": {"bound": "latency (6.4 MFLOP per call: launch and fill dominate)",
                     "achieved": achieved, "peak": roof["peak"], "unit": "TFLOP/s",
                     "frac": achieved / roof["peak"], "peak_source": roof["peak_source"],
                     "kernel": roof["kernel"], "kernel_ms": us / 1e3, "traffic": None},
        "e2e": {"value": e2e_ms * 1e3, "unit": "us per call", "ms_per_step": e2e_ms, "steps": 20,
                "h2d_bytes_per_step": 3 * host[0].numel() * 4,
                "d2h_bytes_per_step": host_out.numel() * 4,
                "path": "AttentionKernel (the demo binding's interface): 12 one-head launches "
                        "through wfattn_attention; q, k, v in one pinned copy, O back"},
        "gpu_launches": args.steps * n_calls, "clocks": clock_info,
    }
    if ctx.rank == 0:
        line["reference_ptx"] = ref_ptx_head_call(ctx, w, q, k, v, args)
    return line


def run_gpt2(args, ctx: Ctx, w: Workload) -> dict:
    """GPT-2 generation tokens/s with every attention through libwfattn (one process per GPU)."""
    torch = ctx.torch
    from warpforth_b200 import gpt2

    dev, world = ctx.dev, ctx.world
    model = gpt2.random_gpt2(seed=1, device=dev)
    prompt = gpt2.synthetic_prompt(32, seed=1)
    prompt_dev = prompt.to(dev)
    restore = gpt2.patch_gpt2()
    steps = max(1, min(args.steps, args.gpt2_steps))
    try:
        for _ in range(args.warmup):
            ids = gpt2.generate(model, prompt_dev, w.S, use_cache=w.use_cache)
        torch.cuda.synchronize()
        calls = gpt2.count_calls(lambda: gpt2.generate(model, prompt_dev, w.S,
                                                       use_cache=w.use_cache))
        total_ms, _, clock_info = time_steps(
            ctx, lambda: gpt2.generate(model, prompt_dev, w.S, use_cache=w.use_cache), steps,
            False)
        ms = ctx.max_over_ranks(total_ms / steps)
        value = w.S * world / (ms / 1e3)
        # end to end: prompt from (pinned) host memory, ids read back, inside the timed region
        host_prompt = prompt.pin_memory()

        def one():
            return gpt2.generate(model, host_prompt.to(dev, non_blocking=True), w.S,
                                 use_cache=w.use_cache).cpu()

        out = one()
        e2e_ms = timed_e2e(ctx, one, min(steps, args.e2e_steps), 0, False)
    finally:
        restore()
    assert ids.shape[1] == 32 + w.S and out.shape[1] == 32 + w.S
    # the attention kernel of the step's largest prefill call, [1, 12, 159, 64] f32, alone
    from warpforth_b200 import warpforth as wf

    s_max = 32 + w.S - 1
    q, k, v = (torch.randn(1, 12, s_max, 64, device=dev) for _ in range(3))
    o = torch.empty_like(q)
    kms = _ref_time(ctx, graph_of(ctx, lambda: wf.attention(q, k, v, out=o)).replay, 100)
    kflops = 4 * 64 * 12 * (s_max * (s_max + 1) // 2)
    roof = f32_roof(ctx, 64)
    peak = roof["peak"]
    line = {
        "metric": "GPT-2 gen tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (random-init weights, random prompt ids)",
        "config": dict(config_of(w, world), device_timing="CUDA events around whole "
                       "generate() calls (host launch path included)"),
        "roofline": {"bound": "launch/latency (attention is a small part of a GPT-2 step)",
                     "kernel": f"{roof['kernel']} at [1,12,{s_max},64]",
                     "achieved": kflops / (kms / 1e3) / 1e12, "peak": peak, "unit": "TFLOP/s",
                     "frac": kflops / (kms / 1e3) / 1e12 / peak, "kernel_ms": kms,
                     "traffic": None, "peak_source": roof["peak_source"],
                     "attention_calls_per_step": calls},
        "e2e": {"value": w.S * world / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                "steps": min(steps, args.e2e_steps),
                "h2d_bytes_per_step": prompt.numel() * prompt.element_size(),
                "d2h_bytes_per_step": out.numel() * out.element_size(),
                "path": "transformers generate -> patched eager_attention_forward -> libwfattn"},
        # library launches per step: one per attention call (two for a decode call)
        "gpu_launches": steps * world * sum(calls.values()) + steps * world * calls.get(
            "decode", 0),
        "clocks": clock_info,
    }
    if ctx.rank == 0 and not w.use_cache:
        line["reference_ptx"] = ref_ptx_gpt2(ctx, w, model, prompt_dev, args)
    return line


# ------------------------------------------------------------------ the reference's compiled kernel
def _ref_kernel():
    from oracle import ref_ptx

    if not ref_ptx.available():
        return None, {"unavailable": "oracle/_ref/attention.ptx missing (make -C oracle ref "
                                     "where the reference tree is present)"}
    return ref_ptx.ReferencePtxKernel(), None


def _ref_time(ctx: Ctx, fn, reps: int) -> float:
    torch = ctx.torch
    fn()
    torch.cuda.synchronize()
    a, b = ctx.event(), ctx.event()
    a.record(ctx.stream)
    for _ in range(reps):
        fn()
    b.record(ctx.stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def ref_ptx_prefill(ctx: Ctx, w: Workload, q, k, v, out, args) -> dict:
    """The reference's compiled kernel on the same f32 inputs: one launch per (batch, head)
    with grid = block = (S, 1, 1), as demo/gpt2_generate.py:42-50 launches it."""
    import numpy as np

    kern, bad = _ref_kernel()
    if bad:
        return bad
    ro = ctx.torch.zeros_like(q)

    def run():
        for b in range(w.B):
            for h in range(w.H):
                kern(q[b, h], k[b, h], v[b, h], ro[b, h], w.S, w.D)

    ms = _ref_time(ctx, run, max(1, min(args.steps, 5)))
    err = float(np.abs(ro.cpu().numpy() - out.cpu().numpy()).max())
    fl = prefill_flops(w)
    return {"value": fl / (ms / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "launches_per_step": w.B * w.H, "max_abs_diff_vs_wfattn": err,
            "what": "demo/attention.ptx (the reference's compiled kernel) via cuModuleLoadData "
                    "+ cuLaunchKernel, one launch per head, timed with CUDA events"}


def ref_ptx_head_call(ctx: Ctx, w: Workload, q, k, v, args) -> dict:
    import numpy as np

    kern, bad = _ref_kernel()
    if bad:
        return bad
    ro = ctx.torch.zeros_like(q)

    def run():
        for h in range(w.H):
            kern(q[0, h], k[0, h], v[0, h], ro[0, h], w.S, w.D)

    ms = _ref_time(ctx, run, 50)
    from warpforth_b200 import warpforth as wf

    err = float(np.abs(ro.cpu().numpy() - wf.attention(q, k, v).cpu().numpy()).max())
    return {"value": ms * 1e3, "unit": "us per call", "launches_per_step": w.H,
            "max_abs_diff_vs_wfattn": err,
            "what": "demo/attention.ptx, 12 one-head launches per call (the demo's loop), "
                    "CUDA events over 50 calls"}


def ref_ptx_gpt2(ctx: Ctx, w: Workload, model, prompt_dev, args) -> dict:
    """The demo's own path: greedy generation with its per-head patch around the compiled
    reference kernel (demo/gpt2_generate.py:25-54)."""
    torch = ctx.torch
    import transformers.models.gpt2.modeling_gpt2 as gpt2_module

    from oracle import ref_ptx
    from warpforth_b200 import gpt2

    kern, bad = _ref_kernel()
    if bad:
        return bad
    original = gpt2_module.eager_attention_forward
    gpt2_module.eager_attention_forward = ref_ptx.make_reference_eager_attn(kern)
    try:
        ids = gpt2.generate(model, prompt_dev, w.S)
        torch.cuda.synchronize()
        a, b = ctx.event(), ctx.event()
        a.record(ctx.stream)
        ids = gpt2.generate(model, prompt_dev, w.S)
        b.record(ctx.stream)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
    finally:
        gpt2_module.eager_attention_forward = original
    restore = gpt2.patch_gpt2()
    try:
        ours = gpt2.generate(model, prompt_dev, w.S)
    finally:
        restore()
    return {"value": w.S / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms,
            "tokens_match_wfattn": bool(torch.equal(ids, ours)),
            "what": "the demo's patch (contiguous copies, zeroed output, one launch per head of "
                    "batch 0) around demo/attention.ptx; one timed generation after one warm-up"}


# ------------------------------------------------------------------ composition
RUNNERS = {"prefill": run_prefill, "decode": run_decode, "gpt2": run_gpt2,
           "head_call": run_head_call}


def summarise_side(line: dict) -> dict:
    keep = ("metric", "value", "unit", "higher_is_better", "ms_per_step", "steps", "warmup",
            "dtype", "config", "roofline", "e2e", "cpu_baseline", "clocks", "gpu_launches",
            "reference_ptx", "parity")
    return {k: line[k] for k in keep if k in line}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["wfattn", "reference"], default="wfattn")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="long_prefill")
    ap.add_argument("--cpu-seconds", type=float, default=6.0,
                    help="target CPU time of each cpu_baseline sample")
    ap.add_argument("--ref-step-seconds", type=float, default=4.0,
                    help="target CPU time of one reference-arm step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-side", action="store_true",
                    help="measure the chosen workload only (no `workloads` object)")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--gpt2-steps", type=int, default=3,
                    help="timed generations of the GPT-2 workloads (at most --steps)")
    ap.add_argument("--shape", default=None,
                    help="B,H,S override of a prefill workload (profiling a smaller case)")
    ap.add_argument("--transport", choices=["auto", "multicast", "peer", "nccl"], default="auto",
                    help="sharded prefill's gather: the kernel writes each output tile once "
                         "through an NVLS multicast address (multicast), stores into every "
                         "rank's buffer over CUDA IPC mappings (peer), or chunked NCCL "
                         "all-gathers; auto takes the first of these that every rank can use")
    ap.add_argument("--chunks", type=int, default=0,
                    help="head chunks per rank for the sharded prefill's gather overlap "
                         "(0: the library default)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    w = WORKLOADS[args.workload]
    if args.shape:
        b, h, s = (int(x) for x in args.shape.split(","))
        if w.kind != "prefill":
            ap.error("--shape applies to prefill workloads only")
        w = replace(w, B=b, H=h, S=s, description=f"causal prefill [{b},{h},{s},{w.D}] "
                    f"{w.dtype} (shape override of {w.name})")
    if args.impl == "reference":
        run_reference(args, w)
        return
    ctx = Ctx()
    if ctx.world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={ctx.world}")
    line = RUNNERS[w.kind](args, ctx, w)
    if ctx.rank == 0 and ctx.world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_of(w, args.cpu_seconds)
    side = {}
    if (ctx.world == 1 and not args.no_side and not args.shape
            and args.workload == "long_prefill"):
        for name in SIDE_WORKLOADS:
            sw = WORKLOADS[name]
            ctx.torch.cuda.empty_cache()
            try:
                sub = RUNNERS[sw.kind](args, ctx, sw)
                if not args.no_cpu_baseline:
                    sub["cpu_baseline"] = cpu_baseline_of(sw, args.cpu_seconds)
                side[name] = summarise_side(sub)
            except Exception as e:  # a side workload never hides the headline line
                side[name] = {"error": f"{type(e).__name__}: {e}"}
    if side:
        line["workloads"] = side
    if ctx.rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()


TRAFFIC_SOURCE = ("dram__bytes_read.sum + dram__bytes_write.sum of one ncu capture of this "
                  "kernel on this workload (profiles/traffic.md), not measured in this run")


def load_traffic(w: Workload):
    """DRAM bytes per launch of the dominant kernel from profiles/traffic.md, if captured."""
    p = ROOT / "profiles" / "traffic.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        cells = [c.strip() for c in line.strip().strip("|").split("|")]
        if len(cells) >= 3 and cells[0] == w.name:
            try:
                return int(cells[2])
            except ValueError:
                return None
    return None


if __name__ == "__main__":
    main()
