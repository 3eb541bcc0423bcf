"""Benchmark of the B200 MoE block (one JSON line on rank 0).

Workload (N=1): one Qwen3-30B-A3B-shaped MoE block (hidden 2048, 128 experts, top-8,
moe_intermediate 768, softmax + top-k renormalisation, 4-bit affine group-64 weights),
decode batch T=64 tokens; synthetic seeded weights and activations with the benchmark
distributions. A step = one block forward over one batch of T tokens; every step uses a
different token batch, and L2 is flushed (a 256 MiB write) before each timed step.

  value  tokens/s, device-timed with CUDA events on the launching stream, inputs
         resident in HBM, block replayed from a CUDA graph (max over ranks)
  e2e    tokens/s through the public API (SparseMoeBlock.forward) from pinned host
         memory: H2D copy of x, block, D2H copy of the output, per step
  roofline  the dominant kernel (largest per-stage device time) against the measured
         HBM copy bandwidth, algorithmic bytes = distinct experts actually selected x
         bytes per expert matrix
  cpu_baseline  the CPU oracle (C restatement of the reference block) on the host cores

--gpus N (under torchrun) runs N ranks; each rank owns T tokens and a full replica of
the block (no data-path collective; weak scaling). --impl reference times the CPU
oracle only (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "MoE-block tokens/s; decode HBM GB/s & prefill TFLOPS vs roofline at 1-8 GPU"
LAUNCHES_PER_STEP = 6  # router, top-k, grouping (one CTA at this size), gate/up, down, combine

# name -> (config attribute of synth, weight seed, tokens, scoring override, bias std, regime)
WORKLOADS = {
    "decode": ("QWEN3_30B_A3B", 1, 64, None, None, "decode"),
    "prefill": ("QWEN3_30B_A3B", 2, 4096, None, None, "prefill"),
    "prefill-skewed": ("QWEN3_30B_A3B", 2, 4096, 1, 2.0, "prefill"),
    "qwen15-prefill": ("QWEN15_MOE_A27B", 0, 512, None, None, "prefill"),
    "qwen15-decode": ("QWEN15_MOE_A27B", 0, 1, None, None, "decode"),
    "lfm2-prefill": ("LFM2_8B_A1B", 3, 1024, None, None, "prefill"),
    "lfm2-decode": ("LFM2_8B_A1B", 3, 1, None, None, "decode"),
}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--workload", default="decode", choices=sorted(WORKLOADS))
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def wait_first_sample(self, timeout=3.0):
        t_end = time.time() + timeout
        while self.proc and time.time() < t_end:
            try:
                if os.path.getsize(self.path) > 0:
                    return
            except OSError:
                pass
            time.sleep(0.05)

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        with open(self.path) as f:
            for line in f:
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    sm.append(float(parts[1]))
                    smax.append(float(parts[2]))
                except ValueError:
                    continue
                for n, v in zip(names, parts[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def make_workload(args, S):
    """(config, host weights, tokens per GPU, regime) of the selected workload."""
    from dataclasses import replace
    name, seed, T, scoring, bias_std, regime = WORKLOADS[args.workload]
    cfg = getattr(S, name)
    if scoring is not None:
        cfg = replace(cfg, scoring=scoring)
    bw = S.host_block(cfg, seed)
    if scoring is not None and bias_std is not None:
        bw = S.with_scoring(bw, scoring, seed, bias_std)
    if args.tokens:
        T = args.tokens
    return bw.config, bw, T, regime


def reference_arm(args):
    """The CPU oracle on this host's cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    import mlx_rs_b200.synth as S
    cfg, bw, T, regime = make_workload(args, S)
    # prefill: each step times a bounded sample of the batch (rows of the block are
    # independent, so the per-token rate of a sample is the rate of the batch)
    Ts = min(T, 128) if regime == "prefill" else T
    xs = [S.host_x(1000 + i, Ts, cfg.hidden) for i in range(4)]
    cores = os.cpu_count() or 1
    for i in range(max(1, min(args.warmup, 2))):
        O.block_forward(bw, xs[i % 4], nthreads=cores)
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        O.block_forward(bw, xs[i % 4], nthreads=cores)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(times)
    value = Ts / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{cfg.name} MoE block {regime}, T={T} tokens", "global_batch": T,
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} block calls of {Ts} of the T={T} tokens (CPU oracle, C "
                                   f"restatement of the reference block; MLX itself is not available)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(bw_host, x_host, seconds):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cores = os.cpu_count() or 1
    T = x_host.shape[0]
    times = []
    t_end = time.perf_counter() + seconds
    while True:
        t0 = time.perf_counter()
        O.block_forward(bw_host, x_host, nthreads=cores)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(times) >= 20:
            break
    ms = 1e3 * statistics.median(times)
    return {"value": T / (ms / 1e3), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{len(times)} block calls of T={T} tokens on the CPU oracle (C restatement of the "
                      f"reference block), median"}


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    import numpy as np
    import torch
    import torch.distributed as dist

    import mlx_rs_b200
    import mlx_rs_b200.synth as S
    from mlx_rs_b200.block import SparseMoeBlock

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    cfg, bw_host, T, regime = make_workload(args, S)
    H = cfg.hidden
    blk = SparseMoeBlock(S.to_device(bw_host, dev), cfg)
    pool = 8
    xs_host = [S.host_x(1000 + 97 * rank + i, T, H) for i in range(pool)]
    xs = [S.x_to_device(x, dev) for x in xs_host]
    blk.reserve(max(T, 64))
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    # warm-up (eager), then capture the block into a CUDA graph fed from a static input
    for i in range(max(3, args.warmup)):
        blk.forward(xs[i % pool], out)
    torch.cuda.synchronize()
    graph = None
    static_x = torch.empty_like(xs[0])
    mode = "eager"
    if not args.no_graph:
        try:
            static_x.copy_(xs[0])
            s = torch.cuda.Stream(dev)
            s.wait_stream(stream)
            with torch.cuda.stream(s):
                blk.forward(static_x, out)
            stream.wait_stream(s)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                blk.forward(static_x, out)
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
            mode = "cuda_graph"
        except Exception as e:  # capture unsupported: time eager launches
            graph = None
            mode = f"eager (graph capture failed: {type(e).__name__})"
            torch.cuda.synchronize()

    def step(i):
        if graph is not None:
            static_x.copy_(xs[i % pool])
            flush.zero_()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            graph.replay()
            b.record(stream)
            return a, b
        flush.zero_()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        blk.forward(xs[i % pool], out)
        b.record(stream)
        return a, b

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    # nvidia-smi samples every 200 ms, longer than the timed steps take, so the sampler
    # runs across a window of back-to-back (untimed) steps that brackets the timed ones.
    clocks = ClockSampler(local)
    clocks.start()
    clocks.wait_first_sample()
    t_busy = time.perf_counter() + 0.6
    while time.perf_counter() < t_busy:
        for i in range(8):
            step(i)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    evs = [step(i) for i in range(args.steps)]
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t_busy = time.perf_counter() + 0.6
    while time.perf_counter() < t_busy:
        for i in range(8):
            step(i)
        torch.cuda.synchronize()
    clock_info = clocks.stop()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    ms = statistics.mean(step_ms)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = world * T / (ms / 1e3)

    # ---- per-stage device times (profile entry point) for the roofline
    stage_acc, n_act = {}, []
    for i in range(max(8, pool)):
        flush.zero_()
        _, st, na = blk.profile(xs[i % pool], out)
        n_act.append(na)
        for kname, v in st.items():
            stage_acc.setdefault(kname, []).append(v)
    stage_ms = {kname: statistics.mean(v) for kname, v in stage_acc.items()}
    U = statistics.mean(n_act)
    wb = S.weight_bytes(cfg)
    per_mat = wb["per_expert"] / 3
    alg = {
        "gate_up": U * 2 * per_mat + T * H * 2,
        "down": U * per_mat + T * cfg.top_k * cfg.moe_inter * 2,
        "router": wb["router"] + T * H * 2,
    }
    P = T * cfg.top_k
    flops = {"gate_up": 2.0 * P * 2 * H * cfg.moe_inter, "down": 2.0 * P * H * cfg.moe_inter}
    dom = max(("gate_up", "down"), key=lambda kname: stage_ms[kname])
    hbm, tf, peak_kind = measured_peaks()
    block_bytes = alg["gate_up"] + alg["down"] + alg["router"]
    if regime == "prefill":
        kind = "tcgen05 grouped GEMM" if T * cfg.top_k >= 32 * cfg.num_experts else "qgemv"
        achieved = flops[dom] / (stage_ms[dom] / 1e3) / 1e12
        roof = {"bound": "tensor", "kernel": f"{kind} {dom}", "achieved": achieved, "peak": tf, "unit": "TFLOP/s",
                "frac": achieved / tf, "peak_kind": f"{peak_kind} bf16 burst", "traffic": None,
                "algorithmic_flops_per_launch": flops[dom], "launch_ms": stage_ms[dom],
                "block_TFLOPs": (flops["gate_up"] + flops["down"]) / (ms / 1e3) / 1e12, "stage_ms": stage_ms}
    else:
        achieved = alg[dom] / (stage_ms[dom] / 1e3) / 1e9
        roof = {"bound": "hbm", "kernel": f"qgemv {dom}", "achieved": achieved, "peak": hbm,
                "unit": "GB/s", "frac": achieved / hbm, "peak_kind": peak_kind,
                "frac_of_8TBps_spec": achieved / 8000.0, "traffic": None,
                "algorithmic_bytes_per_launch": alg[dom], "launch_ms": stage_ms[dom],
                "block_algorithmic_GBps": block_bytes / (ms / 1e3) / 1e9,
                "stage_ms": stage_ms}

    # ---- e2e through the public API from pinned host memory
    xs_pin = [torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).pin_memory() for x in xs_host]
    out_pin = torch.empty(T, H, dtype=torch.bfloat16).pin_memory()
    xdev = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    e2e_ms = []
    for i in range(args.warmup + args.steps):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        xdev.copy_(xs_pin[i % pool], non_blocking=True)
        y = blk.forward(xdev, out)
        out_pin.copy_(y, non_blocking=True)
        b.record(stream)
        b.synchronize()
        if i >= args.warmup:
            e2e_ms.append(a.elapsed_time(b))
    e2e = statistics.mean(e2e_ms)
    if world > 1:
        t = torch.tensor([e2e], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e = float(t.item())

    sweep = {}
    if not args.no_sweep and rank == 0 and world == 1 and regime == "decode" and args.workload == "decode":
        for Ts in (1, 8, 32, 64):
            xsw = [S.device_x(77 + i, Ts, H, dev) for i in range(4)]
            o = torch.empty(Ts, H, dtype=torch.bfloat16, device=dev)
            for i in range(3):
                blk.forward(xsw[i % 4], o)
            tms = []
            for i in range(10):
                flush.zero_()
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                blk.forward(xsw[i % 4], o)
                b.record(stream)
                b.synchronize()
                tms.append(a.elapsed_time(b))
            _, st, na = blk.profile(xsw[0], o)
            bytes_ = na * wb["per_expert"] + wb["router"]
            sweep[f"T{Ts}"] = {"tokens_per_s": Ts / (statistics.median(tms) / 1e3),
                               "ms": statistics.median(tms), "experts": na,
                               "stage_us": {kk: round(vv * 1e3, 2) for kk, vv in st.items()},
                               "block_GBps": bytes_ / (statistics.median(tms) / 1e3) / 1e9}

    cpu = None
    if rank == 0 and world == 1:
        cpu = cpu_baseline(bw_host, xs_host[0][: min(T, 128)], args.cpu_seconds)
        if T > 128:
            cpu["sample"] += f" ({min(T, 128)} of the {T} tokens; rows are independent)"
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{cfg.name} MoE block {regime}, T={T} tokens per GPU", "global_batch": T * world,
                       "seq_len": 1, "parallelism": f"replicas{world}" if world > 1 else "single",
                       "experts": cfg.num_experts, "top_k": cfg.top_k, "hidden": H, "moe_inter": cfg.moe_inter,
                       "l2": "flushed (256 MiB write) before every timed step", "launch": mode,
                       "clock_window": "nvidia-smi every 200 ms across 0.6 s of untimed steps, the timed steps, 0.6 s more",
                       "distinct_experts_per_step": U, "sweep_eager": sweep},
            "roofline": roof,
            "cpu_baseline": cpu,
            "e2e": {"value": world * T / (e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                    "d2h_bytes_per_step": T * H * 2, "ms_per_step": e2e},
            "gpu_launches": LAUNCHES_PER_STEP * args.steps,
            "clocks": clock_info,
            "library": mlx_rs_b200.library_path,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        del graph
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
