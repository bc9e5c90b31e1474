#!/usr/bin/env python
"""Benchmark of the WarpForth attention hot path on B200 (libwfattn).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl wfattn|reference]
                    [--workload long_prefill|prefill|prefill_f32|decode]

For N > 1 launch one process per GPU:
    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P bench.py --gpus N

Workloads (all synthetic, seeded):
  long_prefill (default)  causal prefill [16, 48, 8192, 64] bf16, q/k/v = randn (seed 4);
                          heads split evenly over the N ranks, O all-gathered (NCCL).
                          One step = the whole batch.  Total work is fixed (strong scaling).
  prefill                 causal prefill [8, 12, 1024, 64] bf16, seed 2 (per rank).
  prefill_f32             the same in f32 (the reference-accurate CUDA-core kernel).
  decode                  one-token decode, B=64, H=25, D=64, bf16 cache padded to 4096,
                          kv_lens ~ U[512, 4096] (seed 3); metric = valid KV bytes / s.

Prints ONE JSON line on rank 0.  `value` is device-timed (CUDA events, inputs
resident in HBM, max over ranks); `e2e` repeats the step through the public
API with the inputs copied from pinned host memory and the result read back
inside the timed region.  `--impl reference` times the CPU restatement of the
reference kernel (the oracle, f64, all host threads) on a bounded sample of
the same workload; under torchrun only rank 0 runs it.
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
from dataclasses import dataclass
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


@dataclass(frozen=True)
class Workload:
    name: str
    kind: str  # "prefill" or "decode"
    B: int
    H: int
    S: int
    D: int
    seed: int
    dtype: str  # "bf16" or "f32"
    sharded: bool
    description: str


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
}


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


# ------------------------------------------------------------------ CPU side
def cpu_sample(w: Workload, target_s: float, threads: int) -> dict:
    """Times the oracle (f64 restatement of the reference kernel) on a bounded sample.

    Prefill: the last R query rows of `nh` heads of the workload's shape (the
    costliest rows: each sees all S keys).  Decode: `nb` whole sequences.
    Returns value in the workload's metric unit plus a description.
    """
    import numpy as np
    import torch

    import oracle

    if w.kind == "gpt2":
        return gpt2_cpu_sample(target_s, threads)
    g = torch.Generator().manual_seed(w.seed)

    def bf(t):
        return t.to(torch.bfloat16).float().numpy() if w.dtype == "bf16" else t.numpy()

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
    nb = 4
    reps = 1
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


def run_reference(args, w: Workload) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle

    threads = host_threads()
    metric, unit, hib = metric_of(w)
    vals = []
    sample = None
    for i in range(args.warmup + args.steps):
        r = cpu_sample(w, args.ref_step_seconds, threads)
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
    return "causal SDPA TFLOP/s", "TFLOP/s", True


def config_of(w: Workload, n: int) -> dict:
    cfg = {"workload": w.description, "batch": w.B, "heads": w.H, "head_dim": w.D,
           "seed": w.seed}
    if w.kind == "gpt2":
        cfg.update({"model": "gpt2-small (12 layers, d_model 768, vocab 50257, ctx 1024)",
                    "prompt_len": 32, "new_tokens": w.S, "use_cache": False,
                    "parallelism": f"replicas/{n}" if n > 1 else "single",
                    "l2": "not applicable (end-to-end generation)"})
        return cfg
    if w.kind == "prefill":
        cfg.update({"seq_len": w.S, "causal": True,
                    "parallelism": f"heads/{n}" if w.sharded and n > 1 else
                    (f"replicas/{n}" if n > 1 else "single"),
                    "l2": "inputs larger than L2 (126 MB)" if w.S >= 4096 else
                    "L2 flushed between timed steps (256 MB write)"})
    else:
        cfg.update({"max_kv_len": w.S, "kv_lens": "U[512,4096] seed 3 (sum 142652)",
                    "parallelism": f"replicas/{n}" if n > 1 else "single",
                    "l2": "inputs larger than L2 (913 MB of K/V read per step, 126 MB L2)"})
    return cfg


# ------------------------------------------------------------------ GPU side
def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["wfattn", "reference"], default="wfattn")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="long_prefill")
    ap.add_argument("--cpu-seconds", type=float, default=10.0,
                    help="target CPU time of the cpu_baseline sample")
    ap.add_argument("--ref-step-seconds", type=float, default=4.0,
                    help="target CPU time of one reference-arm step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--shape", default=None,
                    help="B,H,S override of a prefill workload (profiling a smaller case)")
    ap.add_argument("--transport", choices=["auto", "peer", "nccl"], default="auto",
                    help="sharded prefill's gather: the kernel stores into every rank's buffer "
                         "over CUDA IPC mappings (peer) or chunked NCCL all-gathers")
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
        w = Workload(w.name, w.kind, b, h, s, w.D, w.seed, w.dtype, w.sharded,
                     f"causal prefill [{b},{h},{s},{w.D}] {w.dtype} (shape override of "
                     f"{w.name})")
    if args.impl == "reference":
        run_reference(args, w)
        return
    if w.kind == "gpt2":
        run_gpt2(args, w)
        return
    run_gpu(args, w)


def gpt2_cpu_sample(target_s: float, threads: int) -> dict:
    """Stock eager GPT-2 on the host cores (the demo's torch attention), greedy tokens/s."""
    import torch

    from warpforth_b200 import gpt2

    torch.set_num_threads(threads)
    model = gpt2.random_gpt2(seed=1, device="cpu")
    prompt = gpt2.synthetic_prompt(32, seed=1)
    n = 4
    while True:
        t0 = time.perf_counter()
        gpt2.generate(model, prompt, n, use_cache=False)
        dt = time.perf_counter() - t0
        if dt >= 0.5 * target_s or n >= 128:
            break
        n = min(128, max(n + 1, int(n * min(8.0, target_s / max(dt, 1e-3)))))
    return {"value": n / dt, "unit": "tokens/s", "seconds": dt,
            "sample": f"stock eager GPT-2 (torch CPU, {threads} threads): the first {n} greedy "
                      f"tokens of the same prompt in {dt:.2f} s"}


def run_gpt2(args, w: Workload) -> None:
    """GPT-2 generation tokens/s with every attention through libwfattn (one process per GPU)."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    from warpforth_b200 import gpt2

    model = gpt2.random_gpt2(seed=1, device=dev)
    prompt = gpt2.synthetic_prompt(32, seed=1)
    prompt_dev = prompt.to(dev)
    restore = gpt2.patch_gpt2()
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        gpt2.generate(model, prompt_dev, w.S)
    torch.cuda.synchronize()
    barrier()
    clocks = ClockSampler(physical_gpu_indices(world)) if rank == 0 else None
    if clocks:
        clocks.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        ids = gpt2.generate(model, prompt_dev, w.S)
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    clock_info = clocks.stop() if clocks else None
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    assert ids.shape[1] == 32 + w.S
    value = w.S * world / (ms / 1e3)

    # end to end: prompt from (pinned) host memory, ids read back, inside the timed region
    host_prompt = prompt.pin_memory()
    e2e_steps = max(1, min(args.steps, args.e2e_steps))
    e0.record(stream)
    for _ in range(e2e_steps):
        out = gpt2.generate(model, host_prompt.to(dev, non_blocking=True), w.S).cpu()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
    restore()

    # the attention kernel at the step's largest call, [1, 12, 159, 64] f32, on its own
    from warpforth_b200 import warpforth as wf

    s_max = 32 + w.S - 1
    q, k, v = (torch.randn(1, 12, s_max, 64, device=dev) for _ in range(3))
    o = torch.empty_like(q)
    for _ in range(10):
        wf.attention(q, k, v, out=o)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(100):
        wf.attention(q, k, v, out=o)
    a1.record(stream)
    torch.cuda.synchronize()
    kms = a0.elapsed_time(a1) / 100
    kflops = 4 * 64 * 12 * (s_max * (s_max + 1) // 2)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        r = gpt2_cpu_sample(args.cpu_seconds, os.cpu_count() or 1)
        cpu = {"value": r["value"], "unit": r["unit"], "cores": os.cpu_count(),
               "kind": "port", "sample": r["sample"]}
    if rank == 0:
        peak = 148 * 128 * 2 * 1965e6 / 1e12
        achieved = kflops / (kms / 1e3) / 1e12
        line = {
            "metric": "GPT-2 gen tokens/s", "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (random-init weights, random prompt ids)",
            "config": config_of(w, world),
            "roofline": {"bound": "launch/latency (attention is a small part of a GPT-2 step)",
                         "kernel": "prefill_f32_kernel at [1,12,159,64]",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "kernel_ms": kms, "traffic": None,
                         "peak_source": "nominal f32 FMA rate at max SM clock"},
            "cpu_baseline": cpu,
            "e2e": {"value": w.S * world / (e2e_ms / 1e3), "unit": "tokens/s",
                    "ms_per_step": e2e_ms, "steps": e2e_steps,
                    "h2d_bytes_per_step": prompt.numel() * prompt.element_size(),
                    "d2h_bytes_per_step": out.numel() * out.element_size(),
                    "path": "transformers generate -> patched eager_attention_forward -> "
                            "libwfattn"},
            "gpu_launches": args.steps * world * 12 * w.S,
            "clocks": clock_info,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_gpu(args, w: Workload) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    from warpforth_b200 import warpforth as wf
    from warpforth_b200.sharded import ShardedPrefill

    peaks, peak_src = load_peaks()
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)
    # A step whose inputs exceed L2 (126 MB) needs no flush: long prefill and
    # decode (913 MB of K/V per step).  A flush by writes would also leave L2
    # full of dirty lines whose write-back the next step would pay for.
    needs_flush = w.kind == "prefill" and w.S < 4096

    # ---------------- inputs (identical on every rank) and the step
    tdt = torch.bfloat16 if w.dtype == "bf16" else torch.float32
    torch.manual_seed(w.seed)
    sp = None
    if w.kind == "prefill":
        if w.sharded:
            q, k, v = (torch.randn(w.B, w.H, w.S, w.D, device=dev, dtype=tdt) for _ in range(3))
            sp = ShardedPrefill(w.B, w.H, w.S, w.D, dtype=tdt, device=dev,
                                chunks=args.chunks or None, transport=args.transport)
            qs, ks, vs = sp.shard(q), sp.shard(k), sp.shard(v)
            local_heads = sp.local_heads
            units = prefill_flops(w)  # whole job per step
            kernel_flops = prefill_flops(w, local_heads)

            def compute():
                # this rank's heads; the gather of O rides along (peer stores from
                # the kernel, or per-chunk NCCL all-gathers overlapping compute)
                sp(qs, ks, vs)

            def collective():
                pass

            def kernel_only():
                sp.compute_local(qs, ks, vs)
        else:
            q, k, v = (torch.randn(w.B, w.H, w.S, w.D, device=dev).to(tdt) for _ in range(3))
            out = torch.empty_like(q)
            units = prefill_flops(w) * world  # every rank runs one replica
            kernel_flops = prefill_flops(w)

            def compute():
                wf.attention(q, k, v, out=out)

            def collective():
                pass
        unit_scale = 1e12
    else:
        lens = decode_lens().to(dev)
        kc = torch.randn(w.B, w.H, w.S, w.D, device=dev, dtype=tdt)
        vc = torch.randn(w.B, w.H, w.S, w.D, device=dev, dtype=tdt)
        qd = torch.randn(w.B, w.H, w.D, device=dev, dtype=tdt)
        od = torch.empty(w.B, w.H, w.D, device=dev, dtype=torch.float32)
        ws = wf.DecodeWorkspace()
        kv_bytes = int(decode_lens().sum()) * w.H * w.D * 2 * 2
        units = kv_bytes * world
        kernel_flops = kv_bytes

        def compute():
            wf.decode(qd, kc, vc, lens, out=od, workspace=ws)

        def collective():
            pass
        unit_scale = 1e9

    def step():
        compute()
        collective()

    # ---------------- device-timed loop
    for _ in range(args.warmup):
        if needs_flush:
            flush.zero_()
        step()
    torch.cuda.synchronize()
    timed_compute = compute
    if not w.sharded:
        # The step's library call (its kernel launches) captured once and
        # replayed, so the device timing holds the GPU work and not the
        # Python/ctypes launch path; `e2e` below goes through that path.
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            compute()
        torch.cuda.synchronize()
        timed_compute = graph.replay
    barrier()
    clocks = ClockSampler(physical_gpu_indices(world)) if rank == 0 else None
    if clocks:
        clocks.start()
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    total_ms = 0.0
    torch.cuda.synchronize()
    barrier()
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    if needs_flush:
        # flush between steps; steps are timed individually and summed
        for i in range(args.steps):
            flush.zero_()
            kev[i][0].record(stream)
            timed_compute()
            kev[i][1].record(stream)
            collective()
        torch.cuda.synchronize()
        per_step = []
        for i in range(args.steps):
            per_step.append(kev[i][0].elapsed_time(kev[i][1]))
        total_ms = sum(per_step)
    else:
        t_start.record(stream)
        for i in range(args.steps):
            kev[i][0].record(stream)
            timed_compute()
            kev[i][1].record(stream)
            collective()
        t_end.record(stream)
        torch.cuda.synchronize()
        total_ms = t_start.elapsed_time(t_end)
    barrier()
    clock_info = clocks.stop() if clocks else None
    kernel_ms = statistics.mean(kev[i][0].elapsed_time(kev[i][1]) for i in range(args.steps))
    if w.sharded:
        # The timed steps overlap each chunk's all-gather with the next chunk's
        # compute; the roofline's kernel time comes from the kernels alone.
        for i in range(args.steps):
            kev[i][0].record(stream)
            kernel_only()
            kev[i][1].record(stream)
        torch.cuda.synchronize()
        kernel_ms = statistics.mean(kev[i][0].elapsed_time(kev[i][1]) for i in range(args.steps))
        barrier()
    total_ms = max_over_ranks(total_ms)
    kernel_ms_max = max_over_ranks(kernel_ms)
    ms_per_step = total_ms / args.steps
    value = units / (ms_per_step / 1e3) / unit_scale

    # ---------------- end-to-end through the public API with host buffers
    e2e = run_e2e(args, w, world, rank, dev, tdt, barrier, max_over_ranks, wf, sp, units,
                  unit_scale, flush if needs_flush else None)

    # ---------------- CPU baseline (rank 0, N=1 only)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle

        threads = host_threads()
        r = cpu_sample(w, args.cpu_seconds, threads)
        cpu = {"value": r["value"], "unit": r["unit"], "cores": threads, "kind": "port",
               "sample": r["sample"]}

    if rank == 0:
        metric, unit, hib = metric_of(w)
        if w.kind == "prefill":
            peak_key = "bf16_tflops_sustained" if (w.sharded and ms_per_step > 1000) else \
                "bf16_tflops"
            achieved = kernel_flops / (kernel_ms_max / 1e3) / 1e12
            if w.dtype == "f32":
                # CUDA-core f32 FMA peak: 148 SMs x 128 lanes x 2 FLOP x max SM clock
                peak = 148 * 128 * 2 * float(peaks.get("sm_max_mhz", 1965.0)) * 1e6 / 1e12
                roof = {"bound": "fp32-simt", "achieved": achieved, "peak": peak,
                        "unit": "TFLOP/s", "frac": achieved / peak,
                        "peak_source": "nominal f32 FMA rate at max SM clock"}
            else:
                peak = float(peaks[peak_key])
                roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                        "frac": achieved / peak, "peak_source": f"{peak_src} {peak_key}"}
        else:
            achieved = kernel_flops / (kernel_ms_max / 1e3) / 1e9
            peak = float(peaks["hbm_gbs"])
            roof = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "peak_source": f"{peak_src} hbm_gbs"}
        traffic = load_traffic(w)
        if traffic is not None and w.sharded:
            traffic = int(traffic * local_heads / w.H)  # this rank's launch
        roof["traffic"] = traffic
        roof["kernel_ms"] = kernel_ms_max
        line = {
            "metric": metric, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": hib,
            "scaling": "strong" if w.sharded else "weak",
            "vs_baseline": None, "dtype": w.dtype, "data": "synthetic",
            "config": dict(config_of(w, world), **({"gather": sp.transport} if sp else {}),
                           device_timing=(
                "per-rank CUDA events around each step" if w.sharded else
                "CUDA events around each step's library call, replayed from a CUDA graph")),
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": e2e,
            # kernels of this library per timed step, all ranks: decode = split + combine,
            # sharded prefill = one launch per head chunk, otherwise one launch
            "gpu_launches": args.steps * world * (2 if w.kind == "decode" else
                                                  (sp.chunks if sp is not None else 1)),
            "clocks": clock_info,
        }
        print(json.dumps(line), flush=True)
    if sp is not None:
        sp.close()  # collective: unmaps and frees the peer output buffers
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, w, world, rank, dev, tdt, barrier, max_over_ranks, wf, sp, units, unit_scale,
            flush):
    import torch

    stream = torch.cuda.current_stream(dev)
    steps = max(1, min(args.steps, args.e2e_steps))
    g = torch.Generator().manual_seed(w.seed + 1000)
    if w.kind == "prefill":
        heads = sp.local_heads if sp is not None else w.H
        shape = (w.B, heads, w.S, w.D)
        host = [torch.randn(*shape, generator=g).to(tdt).pin_memory() for _ in range(3)]
        dev_in = [torch.empty(shape, dtype=tdt, device=dev) for _ in range(3)]
        if sp is not None:
            res = sp.output_view()
            host_out = torch.empty(tuple(res.shape), dtype=tdt).pin_memory() if rank == 0 else None
        else:
            res = torch.empty(shape, dtype=tdt, device=dev)
            host_out = torch.empty(shape, dtype=tdt).pin_memory()

        def one():
            for h_, d_ in zip(host, dev_in):
                d_.copy_(h_, non_blocking=True)
            if sp is not None:
                sp(*(sp.split_local(t) for t in dev_in))
                if host_out is not None:
                    host_out.copy_(sp.output_view(), non_blocking=True)
            else:
                wf.attention(*dev_in, out=res)
                host_out.copy_(res, non_blocking=True)

        h2d = sum(t.numel() * t.element_size() for t in host)
        d2h = host_out.numel() * host_out.element_size() if host_out is not None else 0
    else:
        # Decode serving: the KV cache is resident state; a step's inputs are the
        # new query token, the new K/V row of every (batch, head) and the lengths.
        lens_d = decode_lens().to(dev)
        shape = (w.B, w.H, w.S, w.D)
        kc = torch.randn(*shape, device=dev, dtype=tdt)
        vc = torch.randn(*shape, device=dev, dtype=tdt)
        q_h, knew_h, vnew_h = (torch.randn(w.B, w.H, w.D, generator=g).to(tdt).pin_memory()
                               for _ in range(3))
        lens_h = decode_lens().pin_memory()
        qd, knew, vnew = (torch.empty((w.B, w.H, w.D), dtype=tdt, device=dev) for _ in range(3))
        lens = torch.empty(w.B, dtype=torch.int32, device=dev)
        od = torch.empty((w.B, w.H, w.D), dtype=torch.float32, device=dev)
        out_h = torch.empty((w.B, w.H, w.D), dtype=torch.float32).pin_memory()
        ws = wf.DecodeWorkspace()
        bidx = torch.arange(w.B, device=dev)

        def one():
            for h_, d_ in ((q_h, qd), (knew_h, knew), (vnew_h, vnew), (lens_h, lens)):
                d_.copy_(h_, non_blocking=True)
            pos = (lens - 1).long()
            kc[bidx, :, pos] = knew
            vc[bidx, :, pos] = vnew
            wf.decode(qd, kc, vc, lens, out=od, workspace=ws)
            out_h.copy_(od, non_blocking=True)

        h2d = 3 * q_h.numel() * q_h.element_size() + lens_h.numel() * 4
        d2h = out_h.numel() * 4
        del lens_d
    for _ in range(args.warmup):
        one()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    tot = 0.0
    for _ in range(steps):
        if flush is not None:
            flush.zero_()
        torch.cuda.synchronize()
        e0.record(stream)
        one()
        e1.record(stream)
        torch.cuda.synchronize()
        tot += e0.elapsed_time(e1)
    barrier()
    ms = max_over_ranks(tot / steps)
    return {"value": units / (ms / 1e3) / unit_scale, "unit": "TFLOP/s" if w.kind == "prefill"
            else "GB/s", "ms_per_step": ms, "steps": steps,
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "path": "warpforth_b200.warpforth (ctypes) -> libwfattn C ABI, pinned host buffers"}


def host_threads() -> int:
    """Host cores this process may run on.  torchrun sets OMP_NUM_THREADS=1 for every rank, so
    the CPU legs pass their thread count explicitly instead of taking OpenMP's default."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


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
