"""GPU tests of expert parallelism: the EP kernels (moe_ep_route / moe_ep_experts /
moe_ep_finish) through the C ABI, and the NCCL orchestration when several GPUs exist.

On one GPU the ranks are emulated: every rank's route and experts calls run on the same
device and the all-gather / all-to-all are done by indexing. Against the single-device
block (moe_block_forward) and the oracle: routing bit-exact; outputs within the parity
tolerance (the EP sum adds per-rank fp32 partial sums, a different association).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

import mlx_rs_b200.synth as S
from parity import ULP_TOL, ULP_TOL_TC, assert_close

pytestmark = pytest.mark.gpu


def _emulate(cfg, seed, T_r, world, x_seed, norm=False, partial_dtype=None):
    import torch
    from gpu_util import dev_bits, make_block, to_dev
    from mlx_rs_b200.ep import CudaEpOps, expert_range, local_weights
    bw_host = S.host_block(cfg, seed)
    bw_dev = S.to_device(bw_host, "cuda")
    blk = make_block(bw_host)
    H, k = cfg.hidden, cfg.top_k
    x_bits = S.host_x(x_seed, world * T_r, H)
    x_all = to_dev(x_bits)
    ops = CudaEpOps()
    shares = [expert_range(cfg.num_experts, world, r) for r in range(world)]
    bound = [ops.bind(local_weights(bw_dev, e0, n), cfg) for e0, n in shares]
    packed = torch.empty(world * T_r, k, dtype=torch.int32, device="cuda")
    for r in range(world):
        ops.route(bound[r], x_all[r * T_r:(r + 1) * T_r].contiguous(), packed[r * T_r:(r + 1) * T_r])
    partials = []
    for r, (e0, n) in enumerate(shares):
        p = torch.empty(world * T_r, H, dtype=partial_dtype or torch.float32, device="cuda")
        ops.experts(bound[r], x_all, packed, e0, n, p)
        partials.append(p)
    out = torch.empty(world * T_r, H, dtype=torch.bfloat16, device="cuda")
    nw = to_dev(S.f32_to_bf16_bits(np.linspace(0.5, 1.5, H, dtype=np.float32))) if norm else None
    normed = torch.empty_like(out) if norm else None
    for r in range(world):
        rows = slice(r * T_r, (r + 1) * T_r)
        received = torch.stack([partials[s][rows] for s in range(world)]).contiguous()
        ops.finish(received, world, out[rows], nw, 1e-6, normed[rows] if norm else None)
    idx, w, _, _ = blk.route(x_all)
    ref = blk.forward(x_all)
    torch.cuda.synchronize()
    pk = dev_bits(packed)
    want = dev_bits(idx).astype(np.uint32) | (dev_bits(w).astype(np.uint32) << 16)
    assert np.array_equal(pk, want.reshape(pk.shape)), "EP routing differs from the block's"
    if norm:
        from mlx_rs_b200 import ops as mops
        ref_norm = mops.fast_rms_norm(out, nw, 1e-6)
        assert np.array_equal(dev_bits(normed), dev_bits(ref_norm)), "fused RMSNorm differs"
    return bw_host, x_bits, dev_bits(out), dev_bits(ref)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ep_decode_qwen3_matches_block_and_oracle(world):
    import oracle as O
    cfg = S.QWEN3_30B_A3B
    bw, x, out, ref = _emulate(cfg, 1, 8, world, 300 + world)
    m = assert_close(out, ref, f"EP world {world} vs block", ULP_TOL)
    assert m["frac_exact"] > 0.99, m
    y, _, _ = O.block_forward(bw, x)
    assert_close(out, y, f"EP world {world} vs oracle", ULP_TOL)


@pytest.mark.parametrize("world", [2, 8])
def test_ep_bf16_partials_qwen3(world):
    """bf16 partial sums through the combine (moe_ep_experts_bf16 / moe_ep_finish_bf16):
    within the tolerance of the single-device block and of the oracle; a token whose
    experts all lie on one rank gets that rank's sum rounded once, as the block does."""
    import oracle as O
    import torch
    cfg = S.QWEN3_30B_A3B
    bw, x, out, ref = _emulate(cfg, 1, 8, world, 320 + world, partial_dtype=torch.bfloat16)
    assert_close(out, ref, f"EP bf16 partials world {world} vs block", ULP_TOL)
    y, _, _ = O.block_forward(bw, x)
    assert_close(out, y, f"EP bf16 partials world {world} vs oracle", ULP_TOL)


def test_ep_lfm2_sigmoid_world2():
    import oracle as O
    cfg = S.LFM2_8B_A1B
    bw, x, out, ref = _emulate(cfg, 3, 6, 2, 310)
    assert_close(out, ref, "EP lfm2 vs block", ULP_TOL)
    y, _, _ = O.block_forward(bw, x)
    assert_close(out, y, "EP lfm2 vs oracle", ULP_TOL)


def test_ep_prefill_tc_path_world2():
    """2048 tokens over 2 ranks: 128 rows per expert, the tcgen05 GEMM under EP grouping."""
    _, _, out, ref = _emulate(S.QWEN3_30B_A3B, 2, 1024, 2, 320)
    m = assert_close(out, ref, "EP prefill vs block", ULP_TOL_TC)
    assert m["frac_exact"] > 0.99, m


def test_ep_fused_norm_bit_exact():
    _emulate(S.QWEN3_30B_A3B, 1, 16, 4, 330, norm=True)


def test_ep_errors():
    import torch
    from mlx_rs_b200._lib import MlxError
    from mlx_rs_b200.ep import CudaEpOps, local_weights
    ops = CudaEpOps()
    cfg = S.QWEN3_30B_A3B
    bw = S.to_device(S.host_block(S.MoeConfig(256, 8, 2, 64, 0, S.SCORING_SOFTMAX, True, False), 5), "cuda")
    b = ops.bind(local_weights(bw, 0, 4), bw.config)
    x = torch.zeros(4, 256, dtype=torch.bfloat16, device="cuda")
    pk = torch.zeros(4, 2, dtype=torch.int32, device="cuda")
    part = torch.zeros(4, 256, dtype=torch.float32, device="cuda")
    with pytest.raises(MlxError) as ei:
        ops.experts(b, x, pk, 6, 4, part)  # experts [6, 10) outside [0, 8)
    assert ei.value.rc == 1
    shared = S.to_device(S.host_block(S.MoeConfig(256, 8, 2, 64, 64, S.SCORING_SOFTMAX, False, True), 6), "cuda")
    with pytest.raises(MlxError) as ei:
        local_weights(shared, 0, 4)
    assert ei.value.rc == 2
    del cfg


# ----------------------------------------------------------------------------------
# real NCCL, when the box has several GPUs
# ----------------------------------------------------------------------------------

def _nccl_worker(rank, world, port, q):
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from gpu_util import dev_bits, make_block
        from mlx_rs_b200.ep import ExpertParallelBlock, ExpertParallelStack, expert_range, local_weights
        cfg = S.QWEN3_30B_A3B
        T_r = 16
        res = {}
        hosts = [S.host_block(cfg, 400 + l) for l in range(2)]
        x_bits = S.host_x(401, world * T_r, cfg.hidden)
        x_all = S.x_to_device(x_bits, dev)
        e0, n = expert_range(cfg.num_experts, world, rank)
        eps = [ExpertParallelBlock(local_weights(S.to_device(h, dev), e0, n), cfg, expert_begin=e0, num_local=n)
               for h in hosts]
        rows = slice(rank * T_r, (rank + 1) * T_r)
        out = eps[0](x_all[rows].contiguous())
        ref = make_block(hosts[0]).forward(x_all)
        torch.cuda.synchronize()
        m = assert_close(dev_bits(out), dev_bits(ref)[rows], f"nccl rank {rank}", ULP_TOL)
        res["frac_exact"] = m["frac_exact"]
        nw = S.x_to_device(S.f32_to_bf16_bits(np.linspace(0.5, 1.5, cfg.hidden, dtype=np.float32)), dev)
        stack = ExpertParallelStack(eps, [None, nw])
        y = stack(x_all[rows].contiguous())
        torch.cuda.synchronize()
        res["stack_finite"] = bool(torch.isfinite(y.float()).all())
        # the same block in two token chunks (collectives overlapped with the experts)
        eps[0].chunks = 2
        out2 = eps[0](x_all[rows].contiguous())
        torch.cuda.synchronize()
        m2 = assert_close(dev_bits(out2), dev_bits(ref)[rows], f"nccl chunked rank {rank}", ULP_TOL)
        res["frac_exact_chunked"] = m2["frac_exact"]
        q.put((rank, "ok", res))
    except Exception:
        import traceback
        q.put((rank, "error", traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def test_ep_nccl_multi_gpu():
    import torch
    import torch.multiprocessing as mp
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("one GPU: the NCCL path needs two or more")
    world = 4 if n >= 4 else 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_nccl_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, st, payload = q.get(timeout=300)
            results[r] = (st, payload)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(world):
        st, payload = results[r]
        assert st == "ok", f"rank {r}:\n{payload}"
        assert payload["frac_exact"] > 0.99 and payload["stack_finite"], payload
        assert payload["frac_exact_chunked"] > 0.99, payload


def test_ep_world8_hybrid_paths():
    """8 ranks, 64 tokens each: ~32 rows per local expert, so experts from 32 rows go to
    the tcgen05 kernel and the smaller ones stay on the GEMV, under the EP grouping."""
    _, _, out, ref = _emulate(S.QWEN3_30B_A3B, 1, 64, 8, 340)
    m = assert_close(out, ref, "EP world 8 hybrid vs block", ULP_TOL_TC)
    assert m["mean_rel"] < 5e-3, m
