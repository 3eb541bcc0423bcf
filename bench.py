"""Benchmark of the B200 MoE block (one JSON line on rank 0).

Default workload (N=1): one Qwen3-30B-A3B-shaped MoE block (hidden 2048, 128 experts,
top-8, moe_intermediate 768, softmax + top-k renormalisation, 4-bit affine group-64
weights), decode batch T=64 tokens; synthetic seeded weights and activations with the
benchmark distributions. A step = one block forward over one batch of T tokens; every
step uses a different token batch, and L2 is flushed (a 256 MiB write) before each
timed step.

  value  tokens/s, device-timed with CUDA events on the launching stream, inputs
         resident in HBM (max over ranks)
  e2e    tokens/s through the public API (SparseMoeBlock.forward, or
         ExpertParallelBlock.forward under torchrun) from pinned host memory: H2D copy
         of x, block, D2H copy of the output, per step; the timed steps are issued back
         to back and the host waits once
  roofline  the dominant kernel (largest per-stage device time) against the measured
         HBM copy bandwidth (decode) or bf16 tensor peak (prefill)
  cpu_baseline  the CPU oracle (C restatement of the reference block) on the host cores

--gpus N (under torchrun, one rank per GPU): expert parallelism. Rank r owns experts
[r*E/N, (r+1)*E/N) and its own T tokens (weak scaling: 64 decode tokens per GPU); the
token rows are all-gathered and the fp32 partial outputs returned with an all-to-all
over NCCL (mlx_rs_b200.ep).
--workload stack-prefill / stack-decode: the 48-block Qwen3-30B-A3B stack with an
RMSNorm between blocks, 8192 / 256 tokens in total split over the N ranks (strong
scaling), expert-parallel for N > 1.
--impl reference times the CPU oracle only (rank 0).
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

# name -> (config attribute of synth, weight seed, tokens, scoring override, bias std, regime, blocks)
# Single blocks: tokens per GPU. Stacks: tokens in total, split over the GPUs.
WORKLOADS = {
    "decode": ("QWEN3_30B_A3B", 1, 64, None, None, "decode", 1),
    "prefill": ("QWEN3_30B_A3B", 2, 4096, None, None, "prefill", 1),
    "prefill-skewed": ("QWEN3_30B_A3B", 2, 4096, 1, 2.0, "prefill", 1),
    "qwen15-prefill": ("QWEN15_MOE_A27B", 0, 512, None, None, "prefill", 1),
    "qwen15-decode": ("QWEN15_MOE_A27B", 0, 1, None, None, "decode", 1),
    "lfm2-prefill": ("LFM2_8B_A1B", 3, 1024, None, None, "prefill", 1),
    "lfm2-decode": ("LFM2_8B_A1B", 3, 1, None, None, "decode", 1),
    "stack-prefill": ("QWEN3_30B_A3B", 4, 8192, None, None, "prefill", 48),
    "stack-decode": ("QWEN3_30B_A3B", 4, 256, None, None, "decode", 48),
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
    ap.add_argument("--ep-partials", choices=("f32", "bf16"), default="f32",
                    help="expert-parallel combine: fp32 partial sums (default) or bf16 (half the bytes)")
    ap.add_argument("--no-configs", action="store_true",
                    help="skip the per-configuration sub-records of the default run")
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


# DRAM traffic per launch of the dominant kernel (dram__bytes_read.sum +
# dram__bytes_write.sum) from one ncu --set full capture of the same workload on a B200.
NCU_TRAFFIC = {
    ("decode", "gate_up"): 215_520_768 + 4_102_656,
    ("decode", "down"): 107_880_960 + 3_843_840,
    ("prefill", "gate_up"): 262_024_704 + 40_618_240,
    ("prefill", "down"): 163_624_704 + 99_390_976,
}


def make_workload(args, S, host=True):
    """(config, host weights of block 0 or None, tokens, regime, blocks) of the workload."""
    from dataclasses import replace
    name, seed, T, scoring, bias_std, regime, layers = WORKLOADS[args.workload]
    cfg = getattr(S, name)
    if scoring is not None:
        cfg = replace(cfg, scoring=scoring)
    bw = None
    if host:
        bw = S.host_block(cfg, seed)
        if scoring is not None and bias_std is not None:
            bw = S.with_scoring(bw, scoring, seed, bias_std)
        cfg = bw.config
    if args.tokens:
        T = args.tokens
    return cfg, bw, T, regime, layers


def workload_config(cfg, regime, T, world, layers, tokens_per_gpu=None):
    """The `config` object of a bench line: the same dict in both arms (b200 and
    reference) for the same workload and GPU count."""
    what = f"stack of {layers} MoE blocks + RMSNorm" if layers > 1 else "MoE block"
    per = "in total" if layers > 1 else "per GPU"
    c = {"workload": f"{cfg.name} {what} {regime}, T={T} tokens {per}",
         "global_batch": T * (world if layers == 1 else 1), "seq_len": 1,
         "parallelism": f"ep{world}" if world > 1 else "single",
         "experts": cfg.num_experts, "top_k": cfg.top_k, "hidden": cfg.hidden, "moe_inter": cfg.moe_inter,
         "shared_inter": cfg.shared_inter,
         "l2": ("inputs larger than L2 (each step streams every block's weights)" if layers > 1
                else "flushed (256 MiB write) before every timed step")}
    if tokens_per_gpu is not None:
        c["tokens_per_gpu"] = tokens_per_gpu
    return c


def parity_metrics(y_bits, ref_bits):
    """Output parity of GPU rows against the oracle's rows for the same tokens (bf16 bit
    patterns): max |diff|, max |diff| / rms(ref), mean relative error, max error in bf16
    ulps of the reference value, share of bit-identical elements."""
    import numpy as np

    def f(b):
        return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    y, r = f(y_bits), f(ref_bits)
    d = np.abs(y - r)
    rms = float(np.sqrt(np.mean(r * r)))
    ulp = 2.0 ** (np.floor(np.log2(np.maximum(np.abs(r), 2.0 ** -126))) - 7)
    return {"max_abs": float(d.max()), "max_abs_over_rms": float(d.max() / rms) if rms else 0.0,
            "mean_rel": float(d.mean() / np.mean(np.abs(r))) if np.any(r) else 0.0,
            "max_ulp": float((d / ulp).max()), "frac_exact": float(np.mean(d == 0)), "rms_ref": rms,
            "tolerance": "mean_rel <= 1e-2 and |diff| <= 2e-2 + 2 (GEMV) or 4 (tcgen05) bf16 ulps of the row's "
                         "largest |value|", "rows": int(np.asarray(ref_bits).shape[0])}


def reference_arm(args):
    """The CPU oracle on this host's cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    import mlx_rs_b200.synth as S
    cfg, bw, T, regime, layers = make_workload(args, S)
    world = args.gpus
    # each step times a bounded sample of one block's tokens (rows of the block are
    # independent, so the per-token rate of a sample is the rate of the batch); a
    # stack's rate is the block rate divided by its number of blocks
    Ts = min(T, 128) if regime == "prefill" or layers > 1 else T
    xs = [S.host_x(1000 + i, Ts, cfg.hidden) for i in range(4)]
    cores = os.cpu_count() or 1
    for i in range(max(1, min(args.warmup, 2))):
        O.block_forward(bw, xs[i % 4], nthreads=cores)
    times = []
    for i in range(args.steps):
        t0 = time.perf_counter()
        O.block_forward(bw, xs[i % 4], nthreads=cores)
        times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.mean(times) * layers
    value = Ts / (ms / 1e3)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong" if layers > 1 else "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(cfg, regime, T, world, layers, T // world if layers > 1 else None),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{args.steps} block calls of {Ts} of the T={T} tokens (CPU oracle, C "
                                   f"restatement of the reference block; MLX itself is not available)"
                                   + (f"; rate divided by the {layers} blocks" if layers > 1 else "")},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def cpu_baseline(bw_host, x_host, seconds, gpu_rows=None):
    """The CPU oracle on this host's cores over the sample x_host (median time of up to
    20 calls within `seconds`). With gpu_rows (the GPU block's output rows for the same
    tokens), the oracle's output of the sample is also the parity reference: adds
    "parity" (parity_metrics) to the record."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cores = os.cpu_count() or 1
    T = x_host.shape[0]
    times = []
    t_end = time.perf_counter() + seconds
    y = None
    while True:
        t0 = time.perf_counter()
        y, _, _ = O.block_forward(bw_host, x_host, nthreads=cores)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end or len(times) >= 20:
            break
    ms = 1e3 * statistics.median(times)
    r = {"value": T / (ms / 1e3), "unit": "tokens/s", "cores": cores, "kind": "port",
         "sample": f"{len(times)} block calls of T={T} tokens on the CPU oracle (C restatement of the "
                   f"reference block), median"}
    if gpu_rows is not None:
        r["parity"] = parity_metrics(gpu_rows, y)
    return r


class Timer:
    """Warm-up, clock sampling window and the timed steps of one bench run.

    step(i) enqueues step i bracketed by two CUDA events on the launching stream and
    returns them. nvidia-smi samples every 200 ms, longer than short steps take, so the
    sampler runs across a window of back-to-back (untimed) steps that brackets the timed
    ones. Returns the mean step time in ms (max over ranks) and the clock record."""

    def __init__(self, args, world, local, dev):
        self.args, self.world, self.local, self.dev = args, world, local, dev

    def _barrier(self):
        import torch
        import torch.distributed as dist
        torch.cuda.synchronize()
        if self.world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def _busy_rounds(self, step, seconds=0.6):
        """Rounds of 4 back-to-back steps that fill `seconds`, agreed by all ranks (every
        rank must run the same number of steps: they hold collectives)."""
        import torch
        import torch.distributed as dist
        t0 = time.perf_counter()
        for i in range(4):
            step(i)
        torch.cuda.synchronize()
        dt = max(time.perf_counter() - t0, 1e-6)
        n = max(1, int(seconds / dt + 0.999))
        if self.world > 1:
            t = torch.tensor([n], device=self.dev, dtype=torch.int64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            n = int(t.item())
        return n

    def _busy(self, step, n):
        import torch
        for _ in range(n):
            for i in range(4):
                step(i)
        torch.cuda.synchronize()

    def run(self, step):
        for i in range(max(3, self.args.warmup)):
            step(i)
        self._barrier()
        n = self._busy_rounds(step)
        self._barrier()
        clocks = ClockSampler(self.local)
        clocks.start()
        clocks.wait_first_sample()
        self._busy(step, n)
        self._barrier()
        evs = [step(i) for i in range(self.args.steps)]
        self._barrier()
        self._busy(step, n)
        self._barrier()
        clock_info = clocks.stop()
        ms = statistics.mean(a.elapsed_time(b) for a, b in evs)
        return self.max_over_ranks(ms), clock_info

    def max_over_ranks(self, v):
        import torch
        import torch.distributed as dist
        if self.world == 1:
            return v
        t = torch.tensor([v], device=self.dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())


def events():
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


class GraphAdapter:
    """A captured torch.cuda.CUDAGraph with its static input and output, used like a
    graph.GraphedForward by e2e_run."""

    def __init__(self, graph, static_x, static_y):
        self.graph, self.static_x, self.static_y = graph, static_x, static_y

    def replay(self):
        self.graph.replay()
        return self.static_y

    def __call__(self, x):
        self.static_x.copy_(x)
        return self.replay()


def e2e_run(args, fwd, xs_host_bits, out_shape, dev, timer, graphed=None):
    """ms per step of H2D (pinned) + forward + D2H, max over ranks: the K steps are issued
    back to back on the stream, each with its own host-to-device copy of that step's
    tokens and device-to-host copy of its output, and the host waits once at the end (a
    serving loop that does not stall the GPU between steps; per-step synchronisation
    would add the host's submission latency to every step). With `graphed` (a
    graph.GraphedForward), each step copies the host tokens straight into its input
    buffer and replays it: the public decode-step API."""
    import numpy as np
    import torch
    stream = torch.cuda.current_stream(dev)
    xs_pin = [torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).pin_memory() for x in xs_host_bits]
    outs_pin = [torch.empty(*out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(args.steps)]
    xdev = graphed.static_x if graphed is not None else torch.empty(xs_pin[0].shape, dtype=torch.bfloat16,
                                                                     device=dev)

    if graphed is not None:
        return e2e_pipelined(args, graphed, xs_pin, outs_pin, dev, timer)

    def step(i, out_pin):
        xdev.copy_(xs_pin[i % len(xs_pin)], non_blocking=True)
        y = fwd(xdev)
        out_pin.copy_(y, non_blocking=True)

    for i in range(args.warmup):
        step(i, outs_pin[0])
    torch.cuda.synchronize(dev)
    a, b = events()
    a.record(stream)
    for i in range(args.steps):
        step(args.warmup + i, outs_pin[i])
    b.record(stream)
    b.synchronize()
    return timer.max_over_ranks(a.elapsed_time(b) / args.steps)


def e2e_pipelined(args, graphed, xs_pin, outs_pin, dev, timer):
    """e2e through a graph.GraphedForward with the copies overlapped with compute: step
    i's tokens go host -> device on an upload stream into one of two staging buffers while
    step i-1 computes; the compute stream copies them into the graph's input, replays, and
    copies the output into one of two output stages, which a download stream copies to the
    step's pinned host buffer. Every step still moves its tokens up and its output down."""
    import torch
    comp = torch.cuda.current_stream(dev)
    up, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    xdev, ydev = graphed.static_x, graphed.static_y
    stage = [torch.empty_like(xdev) for _ in range(2)]
    ostage = [torch.empty_like(ydev) for _ in range(2)]

    def run(n, first, outs):
        ev = lambda: torch.cuda.Event()  # noqa: E731
        h_ev, c_ev, d_ev = [ev() for _ in range(n)], [ev() for _ in range(n)], [ev() for _ in range(n)]

        def upload(i):
            with torch.cuda.stream(up):
                if i >= 2:
                    up.wait_event(c_ev[i - 2])  # step i-2 has read stage[i % 2]
                stage[i % 2].copy_(xs_pin[(first + i) % len(xs_pin)], non_blocking=True)
                h_ev[i].record(up)

        upload(0)
        if n > 1:
            upload(1)
        for i in range(n):
            comp.wait_event(h_ev[i])
            xdev.copy_(stage[i % 2], non_blocking=True)
            y = graphed.replay()
            if i >= 2:
                comp.wait_event(d_ev[i - 2])  # the output stage is free again
            ostage[i % 2].copy_(y, non_blocking=True)
            c_ev[i].record(comp)
            with torch.cuda.stream(down):
                down.wait_event(c_ev[i])
                outs[i].copy_(ostage[i % 2], non_blocking=True)
                d_ev[i].record(down)
            if i + 2 < n:
                upload(i + 2)
        return d_ev[n - 1]

    run(max(1, args.warmup), 0, [outs_pin[0]] * max(1, args.warmup))
    torch.cuda.synchronize(dev)
    a, _ = events()
    a.record(comp)
    up.wait_stream(comp)
    last = run(args.steps, args.warmup, outs_pin)
    b = torch.cuda.Event(enable_timing=True)
    down.wait_event(last)
    b.record(down)
    b.synchronize()
    ms = a.elapsed_time(b) / args.steps
    # the pipelined outputs are the steps' own: first and last timed step against a
    # synchronous replay of the same tokens, bit for bit
    for i in (0, args.steps - 1):
        want = graphed(xs_pin[(args.warmup + i) % len(xs_pin)].to(dev)).cpu()
        if not torch.equal(want.view(torch.int16), outs_pin[i].view(torch.int16)):
            raise RuntimeError(f"pipelined e2e: step {i} output differs from a synchronous replay")
    return timer.max_over_ranks(ms)


def hbm_roofline(name, alg_bytes, launch_ms, extra=None):
    hbm, _, peak_kind = measured_peaks()
    achieved = alg_bytes / (launch_ms / 1e3) / 1e9
    r = {"bound": "hbm", "kernel": name, "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
         "peak_kind": peak_kind, "frac_of_8TBps_spec": achieved / 8000.0, "traffic": None,
         "algorithmic_bytes_per_launch": alg_bytes, "launch_ms": launch_ms}
    r.update(extra or {})
    return r


def tensor_roofline(name, flops, launch_ms, extra=None):
    _, tf, peak_kind = measured_peaks()
    achieved = flops / (launch_ms / 1e3) / 1e12
    r = {"bound": "tensor", "kernel": name, "achieved": achieved, "peak": tf, "unit": "TFLOP/s",
         "frac": achieved / tf, "peak_kind": f"{peak_kind} bf16 burst", "traffic": None,
         "algorithmic_flops_per_launch": flops, "launch_ms": launch_ms}
    r.update(extra or {})
    return r


def capture_graph(fn, static_x, dev, world):
    """CUDA graph of fn(static_x) (collectives included), or None; every rank ends with
    the same choice (a capture that failed on any rank is dropped on all)."""
    import torch
    import torch.distributed as dist
    cur = torch.cuda.current_stream(dev)
    graph, err = None, None
    try:
        s = torch.cuda.Stream(dev)
        s.wait_stream(cur)
        with torch.cuda.stream(s):
            for _ in range(2):
                fn(static_x)
        cur.wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn(static_x)
        torch.cuda.synchronize()
    except Exception as e:
        graph, err = None, f"{type(e).__name__}: {str(e)[:120]}"
        torch.cuda.synchronize()
    if world > 1:
        ok = torch.tensor([0 if graph is None else 1], device=dev, dtype=torch.int32)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok.item()) == 0:
            graph = None
            err = err or "capture failed on another rank"
    if graph is not None:
        graph.replay()
        torch.cuda.synchronize()
    return graph, ("cuda_graph" if graph is not None else f"eager (graph capture failed: {err})")


def group_launches(P, E):
    return 1 if (P <= 32768 and E <= 512) else 3


def main():
    args = parse()
    if args.impl == "reference":
        reference_arm(args)
        return
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        if WORKLOADS[args.workload][6] > 1:
            line = run_stack(args, world, rank, local, dev)
        elif world > 1:
            line = run_ep_block(args, world, rank, local, dev)
        else:
            line = run_block(args, dev)
        if rank == 0:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            torch.cuda.synchronize()
            dist.barrier()
            dist.destroy_process_group()


# Sub-records of the default run: every benchmark configuration that fits one GPU, as
# (label, workload, tokens). The headline line is the Qwen3-30B-A3B decode block at T=64.
CONFIG_RECORDS = [
    ("C0 Qwen1.5-MoE-A2.7B decode T=1", "qwen15-decode", 1),
    ("C0 Qwen1.5-MoE-A2.7B prefill T=512", "qwen15-prefill", 512),
    ("C1 Qwen3-30B-A3B decode T=1", "decode", 1),
    ("C1 Qwen3-30B-A3B decode T=8", "decode", 8),
    ("C1 Qwen3-30B-A3B decode T=32", "decode", 32),
    ("C2 Qwen3-30B-A3B prefill T=4096, uniform routing", "prefill", 4096),
    ("C2 Qwen3-30B-A3B prefill T=4096, skewed routing", "prefill-skewed", 4096),
    ("C3 LFM2-8B-A1B decode T=1", "lfm2-decode", 1),
    ("C3 LFM2-8B-A1B prefill T=1024", "lfm2-prefill", 1024),
]


def block_roofline(cfg, regime, T, stage_ms, U, ms):
    """Roofline of one block run: the dominant expert kernel (decode: algorithmic bytes
    of the distinct experts selected ÷ its device time, against HBM; prefill: 2·P·N·K ÷
    its device time, against the bf16 burst peak) and the whole block's fraction."""
    H, I, k = cfg.hidden, cfg.moe_inter, cfg.top_k
    import mlx_rs_b200.synth as S
    wb = S.weight_bytes(cfg)
    per_mat = wb["per_expert"] / 3
    P = T * k
    alg = {"gate_up": U * 2 * per_mat + T * H * 2, "down": U * per_mat + P * I * 2}
    flops = {"gate_up": 2.0 * P * 2 * H * I, "down": 2.0 * P * H * I}
    shared_flops = 2.0 * T * 3 * H * cfg.shared_inter
    dom = max(("gate_up", "down"), key=lambda kk: stage_ms[kk])
    block_bytes = alg["gate_up"] + alg["down"] + wb["router"] + wb["shared"] + T * H * 2
    block_flops = flops["gate_up"] + flops["down"] + 2.0 * T * cfg.num_experts * H + shared_flops
    hbm, tf, _ = measured_peaks()
    extra = {"stage_ms": stage_ms, "block_ms": ms,
             "block_algorithmic_GBps": block_bytes / (ms / 1e3) / 1e9,
             "block_hbm_frac": block_bytes / (ms / 1e3) / 1e9 / hbm,
             "block_TFLOPs": block_flops / (ms / 1e3) / 1e12,
             "block_tensor_frac": block_flops / (ms / 1e3) / 1e12 / tf}
    if regime == "prefill":
        kind = "tcgen05 grouped GEMM" if P >= 32 * cfg.num_experts else "qgemv"
        return tensor_roofline(f"{kind} {dom}", flops[dom], stage_ms[dom], extra)
    if stage_ms["down"] == 0.0 and stage_ms["router"] == 0.0:
        # the one-launch decode kernel: its whole time is booked as the gate/up stage
        return hbm_roofline("decode_block_kernel (whole block, one launch)", block_bytes, stage_ms["gate_up"], extra)
    return hbm_roofline(f"qgemv {dom}", alg[dom], stage_ms[dom], extra)


def config_records(args, dev, flush, cpu_seconds=2.0):
    """One record per CONFIG_RECORDS entry: tokens/s of the block replayed from a CUDA
    graph (CUDA events around each replay, L2 flushed before each), the roofline of its
    dominant kernel and of the whole block, the CPU oracle on a token sample, and the
    parity of the GPU rows of that sample against the oracle's."""
    import torch

    import mlx_rs_b200.synth as S
    from mlx_rs_b200.block import SparseMoeBlock

    recs = []
    stream = torch.cuda.current_stream(dev)
    cache = {}
    for label, wl, T in CONFIG_RECORDS:
        sub = argparse.Namespace(**vars(args))
        sub.workload, sub.tokens = wl, T
        key = WORKLOADS[wl][:5]
        if key not in cache:
            cache.clear()
            torch.cuda.empty_cache()
            cfg, bw_host, _, regime, _ = make_workload(sub, S)
            cache[key] = (cfg, bw_host, SparseMoeBlock(S.to_device(bw_host, dev), cfg))
        cfg, bw_host, blk = cache[key]
        regime = WORKLOADS[wl][5]
        H = cfg.hidden
        xs_host = [S.host_x(2000 + i, T, H) for i in range(4)]
        xs = [S.x_to_device(x, dev) for x in xs_host]
        blk.reserve(T)
        out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        static_x = xs[0].clone()
        for i in range(3):
            blk.forward(xs[i % 4], out)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            blk.forward(static_x, out)
        times = []
        for i in range(max(3, args.warmup) + args.steps):
            static_x.copy_(xs[i % 4])
            flush.zero_()
            a, b = events()
            a.record(stream)
            g.replay()
            b.record(stream)
            if i >= max(3, args.warmup):
                times.append((a, b))
        torch.cuda.synchronize()
        ms = statistics.mean(a.elapsed_time(b) for a, b in times)
        del g
        stage_acc, n_act = {}, []
        for i in range(4):
            flush.zero_()
            _, st, na = blk.profile(xs[i % 4], out)
            n_act.append(na)
            for kk, v in st.items():
                stage_acc.setdefault(kk, []).append(v)
        stage_ms = {kk: statistics.mean(v) for kk, v in stage_acc.items()}
        roof = block_roofline(cfg, regime, T, stage_ms, statistics.mean(n_act), ms)
        n_s = min(T, 32)
        gpu_rows = S.bf16_tensor_to_bits(blk.forward(xs[0], out)[:n_s])
        cpu = cpu_baseline(bw_host, xs_host[0][:n_s], cpu_seconds, gpu_rows)
        if T > n_s:
            cpu["sample"] += f" ({n_s} of the {T} tokens; rows are independent)"
        recs.append({"config": label, "workload": wl, "tokens": T, "value": T / (ms / 1e3), "unit": "tokens/s",
                     "ms_per_step": ms, "launch": "cuda_graph", "distinct_experts": statistics.mean(n_act),
                     "roofline": roof, "parity": cpu.pop("parity"), "cpu_baseline": cpu})
    cache.clear()
    torch.cuda.empty_cache()
    return recs


def run_block(args, dev):
    """One GPU, one block: device time from a CUDA graph, stage profile, e2e, sweep."""
    import numpy as np
    import torch

    import mlx_rs_b200
    import mlx_rs_b200.synth as S
    from mlx_rs_b200.block import SparseMoeBlock

    cfg, bw_host, T, regime, _ = make_workload(args, S)
    H = cfg.hidden
    blk = SparseMoeBlock(S.to_device(bw_host, dev), cfg)
    pool = 8
    xs_host = [S.host_x(1000 + i, T, H) for i in range(pool)]
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
        a, b = events()
        if graph is not None:
            static_x.copy_(xs[i % pool])
            flush.zero_()
            a.record(stream)
            graph.replay()
            b.record(stream)
            return a, b
        flush.zero_()
        a.record(stream)
        blk.forward(xs[i % pool], out)
        b.record(stream)
        return a, b

    timer = Timer(args, 1, int(dev.index), dev)
    ms, clock_info = timer.run(step)
    value = T / (ms / 1e3)

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
    block_bytes = alg["gate_up"] + alg["down"] + alg["router"]
    if regime == "prefill":
        kind = "tcgen05 grouped GEMM" if P >= 32 * cfg.num_experts else "qgemv"
        roof = tensor_roofline(f"{kind} {dom}", flops[dom], stage_ms[dom],
                               {"block_TFLOPs": (flops["gate_up"] + flops["down"]) / (ms / 1e3) / 1e12,
                                "stage_ms": stage_ms})
    else:
        roof = hbm_roofline(f"qgemv {dom}", alg[dom], stage_ms[dom],
                            {"block_algorithmic_GBps": block_bytes / (ms / 1e3) / 1e9, "stage_ms": stage_ms})
    if not args.tokens and (args.workload, dom) in NCU_TRAFFIC:
        roof["traffic"] = NCU_TRAFFIC[(args.workload, dom)]
        roof["traffic_source"] = "ncu --set full capture of this workload (one launch)"

    # end to end through the public API: the block captured once (graph.GraphedForward)
    # and replayed per step, host tokens in and the step's output back every step
    e2e_api = ("graph.GraphedForward(SparseMoeBlock.forward), pinned H2D + replay + D2H per step, "
               "the copies of neighbouring steps overlapped with compute on upload / download streams")
    graphed = None
    if not args.no_graph:
        try:
            from mlx_rs_b200.graph import GraphedForward
            out_g = torch.empty_like(out)
            graphed = GraphedForward(lambda xd: blk.forward(xd, out_g), xs[0])
        except Exception as ex:  # eager public API instead
            graphed = None
            e2e_api = f"SparseMoeBlock.forward eager (graph capture failed: {type(ex).__name__})"
    if graphed is None and args.no_graph:
        e2e_api = "SparseMoeBlock.forward eager, pinned H2D + forward + D2H per step, steps issued back to back"
    e2e = e2e_run(args, lambda xd: blk.forward(xd, out), xs_host, (T, H), dev, timer, graphed)

    sweep = {}
    if not args.no_sweep and regime == "decode" and args.workload == "decode":
        for Ts in (1, 8, 32, 64):
            xsw = [S.device_x(77 + i, Ts, H, dev) for i in range(4)]
            o = torch.empty(Ts, H, dtype=torch.bfloat16, device=dev)
            for i in range(3):
                blk.forward(xsw[i % 4], o)
            tms = []
            for i in range(10):
                flush.zero_()
                a, b = events()
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

    n_s = min(T, 128)
    gpu_rows = S.bf16_tensor_to_bits(blk.forward(xs[0], out)[:n_s])
    cpu = cpu_baseline(bw_host, xs_host[0][:n_s], args.cpu_seconds, gpu_rows)
    if T > 128:
        cpu["sample"] += f" ({n_s} of the {T} tokens; rows are independent)"
    launches = 5 + group_launches(P, cfg.num_experts) + (2 if cfg.shared_inter else 0)
    configs = []
    if args.workload == "decode" and not args.tokens and not args.no_configs:
        del bw_host
        configs = config_records(args, dev, flush)
    return {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(cfg, regime, T, 1, 1),
        "details": {"launch": mode,
                    "clock_window": "nvidia-smi every 200 ms across 0.6 s of untimed steps, the timed steps, "
                                    "0.6 s more",
                    "distinct_experts_per_step": U, "sweep_eager": sweep},
        "roofline": roof,
        "parity": cpu.get("parity"),
        "cpu_baseline": cpu,
        "configs": configs,
        "e2e": {"value": T / (e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2, "ms_per_step": e2e, "api": e2e_api},
        "gpu_launches": launches * args.steps,
        "clocks": clock_info,
        "library": mlx_rs_b200.library_path,
    }


def ep_stage_times(blk, x, dev, world, reps=6):
    """Device time of each step of an expert-parallel block (the all-gather of the token
    rows, the route of all gathered tokens, experts, the all-to-all, finish), from CUDA
    events between the steps."""
    import torch
    import torch.distributed as dist
    b = blk.buffers(x.shape[0], dev)
    out = torch.empty_like(x)
    names = ("all_gather", "route", "experts", "all_to_all", "finish")
    acc = {n: [] for n in names}
    stream = torch.cuda.current_stream(dev)
    for _ in range(reps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
        ev[0].record(stream)
        dist.all_gather_into_tensor(b.x_all.view(torch.uint8), x.view(torch.uint8))
        ev[1].record(stream)
        blk.ops.route(blk.bound, b.x_all, b.packed_all)
        ev[2].record(stream)
        blk.ops.experts(blk.bound, b.x_all, b.packed_all, blk.expert_begin, blk.num_local, b.partial)
        ev[3].record(stream)
        dist.all_to_all_single(b.received.view(-1), b.partial.view(-1))
        ev[4].record(stream)
        blk.ops.finish(b.received, world, out)
        ev[5].record(stream)
        torch.cuda.synchronize()
        for i, n in enumerate(names):
            acc[n].append(ev[i].elapsed_time(ev[i + 1]))
    return {n: statistics.median(v) for n, v in acc.items()}, b


def local_active_experts(b, e0, n):
    import numpy as np
    pk = b.packed_all.cpu().numpy().view(np.uint32) & 0xFFFF
    loc = pk[(pk >= e0) & (pk < e0 + n)]
    return int(np.unique(loc).size), int(loc.size)


def run_ep_block(args, world, rank, local, dev):
    """N ranks, one block, expert-parallel; each rank brings its own T tokens."""
    import torch

    import mlx_rs_b200
    import mlx_rs_b200.synth as S
    from mlx_rs_b200.ep import ExpertParallelBlock, expert_range, local_weights

    cfg, bw_host, T, regime, _ = make_workload(args, S)
    H = cfg.hidden
    e0, n = expert_range(cfg.num_experts, world, rank)
    blk = ExpertParallelBlock(local_weights(S.to_device(bw_host, dev), e0, n), cfg, expert_begin=e0, num_local=n,
                              partials=args.ep_partials)
    del bw_host
    pool = 8
    xs_host = [S.host_x(1000 + 97 * rank + i, T, H) for i in range(pool)]
    xs = [S.x_to_device(x, dev) for x in xs_host]
    out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    static_x = torch.empty_like(xs[0])
    static_x.copy_(xs[0])
    graph, mode = (None, "eager") if args.no_graph else capture_graph(lambda x: blk.forward(x, out), static_x,
                                                                        dev, world)

    def step(i):
        a, b = events()
        flush.zero_()
        if graph is not None:
            static_x.copy_(xs[i % pool])
            a.record(stream)
            graph.replay()
        else:
            a.record(stream)
            blk.forward(xs[i % pool], out)
        b.record(stream)
        return a, b

    timer = Timer(args, world, local, dev)
    ms, clock_info = timer.run(step)
    value = world * T / (ms / 1e3)

    stage_ms, buf = ep_stage_times(blk, xs[0], dev, world)
    n_act, n_pairs = local_active_experts(buf, e0, n)
    wb = S.weight_bytes(cfg)
    P_all = world * T * cfg.top_k
    flops = 2.0 * n_pairs * 3 * H * cfg.moe_inter
    if regime == "prefill":
        roof = tensor_roofline("ep experts (gate/up + down)", flops, stage_ms["experts"], {"stage_ms": stage_ms})
    else:
        roof = hbm_roofline("ep experts (gate/up + down)", n_act * wb["per_expert"], stage_ms["experts"],
                            {"stage_ms": stage_ms, "local_experts_touched": n_act})
    roof["rank"] = 0  # rank 0's own experts and their device time
    # e2e through the captured block (its NCCL calls inside) when there is one
    e2e = e2e_run(args, lambda xd: blk.forward(xd, out), xs_host, (T, H), dev, timer,
                  GraphAdapter(graph, static_x, out) if graph is not None else None)
    del graph  # holds NCCL work: released before the process group is destroyed
    launches = 4 + 2 + group_launches(P_all, n)
    return {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(cfg, regime, T, world, 1),
        "details": {"experts_per_gpu": n, "collectives": "NCCL all_gather of the token rows (dispatch; every rank routes all gathered tokens), all_to_all (combine)", "ep_partials": args.ep_partials,
                    "launch": mode,
                    "clock_window": "nvidia-smi every 200 ms across 0.6 s of untimed steps, the timed steps, "
                                    "0.6 s more"},
        "roofline": roof,
        "cpu_baseline": None,
        "e2e": {"value": world * T / (e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": T * H * 2,
                "d2h_bytes_per_step": T * H * 2, "ms_per_step": e2e},
        "gpu_launches": launches * args.steps,
        "clocks": clock_info,
        "library": mlx_rs_b200.library_path,
    }


def run_stack(args, world, rank, local, dev):
    """The 48-block stack, T tokens in total over the N ranks (strong scaling)."""
    import numpy as np
    import torch

    import mlx_rs_b200
    import mlx_rs_b200.synth as S
    from mlx_rs_b200.block import MoeStack, RmsNorm, SparseMoeBlock
    from mlx_rs_b200.ep import ExpertParallelBlock, ExpertParallelStack, expert_range, local_weights

    cfg, _, T, regime, layers = make_workload(args, S, host=False)
    seed = WORKLOADS[args.workload][1]
    H = cfg.hidden
    if T % world:
        raise SystemExit(f"{T} tokens do not split over {world} ranks")
    T_r = T // world
    e0, n = expert_range(cfg.num_experts, world, rank)
    ones = torch.ones(H, dtype=torch.bfloat16, device=dev)
    blocks = []
    for l in range(layers):
        bw = S.device_block(cfg, seed * 1000 + l, dev)  # identical on every rank
        if world > 1:
            blocks.append(ExpertParallelBlock(local_weights(bw, e0, n), cfg, expert_begin=e0, num_local=n,
                                              partials=args.ep_partials))
        else:
            blocks.append(SparseMoeBlock(bw, cfg))
        del bw
    torch.cuda.empty_cache()
    if world > 1:
        stack = ExpertParallelStack(blocks, [None] + [ones] * (layers - 1))
    else:
        for b in blocks:
            b.reserve(T)
        stack = MoeStack(blocks, [None] + [RmsNorm(ones, 1e-6)] * (layers - 1))
    pool = 4
    xs = [S.device_x(seed * 7 + i, T, H, dev)[rank * T_r:(rank + 1) * T_r].contiguous() for i in range(pool)]
    out = torch.empty(T_r, H, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)

    def fwd(x):
        return stack.forward(x, out) if world > 1 else out.copy_(stack.forward(x))

    # the whole stack (collectives included) replays from one CUDA graph
    static_x = torch.empty_like(xs[0])
    static_x.copy_(xs[0])
    graph, mode = (None, "eager") if args.no_graph else capture_graph(fwd, static_x, dev, world)

    def step(i):
        a, b = events()
        if graph is not None:
            static_x.copy_(xs[i % pool])
            a.record(stream)
            graph.replay()
            b.record(stream)
            return a, b
        a.record(stream)
        fwd(xs[i % pool])
        b.record(stream)
        return a, b

    timer = Timer(args, world, local, dev)
    ms, clock_info = timer.run(step)
    value = T / (ms / 1e3)

    # roofline: the dominant kernel of one block of this rank's share
    wb = S.weight_bytes(cfg)
    if world > 1:
        stage_ms, buf = ep_stage_times(blocks[0], xs[0], dev, world)
        n_act, n_pairs = local_active_experts(buf, e0, n)
        flops = 2.0 * n_pairs * 3 * H * cfg.moe_inter
        kname, launch_ms, bytes_ = "ep experts (gate/up + down)", stage_ms["experts"], n_act * wb["per_expert"]
    else:
        _, stage_ms, n_act = blocks[0].profile(xs[0])
        P = T * cfg.top_k
        dom = max(("gate_up", "down"), key=lambda k: stage_ms[k])
        mats = 2 if dom == "gate_up" else 1
        flops = 2.0 * P * mats * H * cfg.moe_inter
        bytes_ = n_act * wb["per_expert"] * mats / 3
        kname = f"{'tcgen05 grouped GEMM' if P >= 32 * cfg.num_experts else 'qgemv'} {dom}"
        launch_ms = stage_ms[dom]
    extra = {"stage_ms_block0": stage_ms, "stack_ms": ms, "rank": 0}
    if regime == "prefill":
        roof = tensor_roofline(kname, flops, launch_ms, extra)
    else:
        roof = hbm_roofline(kname, bytes_, launch_ms, dict(extra, experts_touched=n_act))

    xs_host = [S.bf16_tensor_to_bits(x) for x in xs[:2]]
    e2e = e2e_run(args, fwd, xs_host, (T_r, H), dev, timer)
    del graph  # holds NCCL work: released before the process group is destroyed
    cpu = None
    if rank == 0 and world == 1:
        bw0 = S.host_block(cfg, 1)
        cpu = cpu_baseline(bw0, S.host_x(5, 128, H), min(args.cpu_seconds, 8.0))
        cpu["value"] /= layers
        cpu["sample"] += f" of one block, rate divided by the {layers} blocks"
    P_all = T * cfg.top_k
    if world > 1:
        per_block = 4 + 2 + group_launches(P_all, n)
    else:
        per_block = 5 + group_launches(P_all, cfg.num_experts) + 1  # + RMSNorm
    return {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload_config(cfg, regime, T, world, layers, T_r),
        "details": {"experts_per_gpu": n, "launch": mode,
                    "clock_window": "nvidia-smi every 200 ms across 0.6 s of untimed steps, the timed steps, "
                                    "0.6 s more"},
        "roofline": roof,
        "cpu_baseline": cpu,
        "e2e": {"value": T / (e2e / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": T_r * H * 2,
                "d2h_bytes_per_step": T_r * H * 2, "ms_per_step": e2e},
        "gpu_launches": per_block * layers * args.steps,
        "clocks": clock_info,
        "library": mlx_rs_b200.library_path,
    }


if __name__ == "__main__":
    main()
