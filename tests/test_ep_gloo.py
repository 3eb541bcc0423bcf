"""Expert-parallel orchestration (mlx_rs_b200.ep) over gloo ranks on CPU.

The compute steps run on the CPU oracle (tests/ep_oracle_ops.py); what is under test
is the orchestration: expert ranges, token ownership, the all-gather dispatch, the
equal-part all-to-all combine and the rank-order finish. Against the single-device
block of the oracle: routing bit-exact; outputs within the parity tolerance (they
differ only by the fp32 association of the k-term sum, in practice not at all).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import mlx_rs_b200.synth as S

CFG = S.MoeConfig(256, 8, 4, 128, 0, S.SCORING_SOFTMAX, True, False, name="ep-small")
CFG_SIG = S.MoeConfig(256, 8, 2, 64, 0, S.SCORING_SIGMOID_BIAS_SELECT, True, False, name="ep-sigmoid")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, case, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle as O
        from ep_oracle_ops import OracleEpOps, bits, from_bits, local_block
        from mlx_rs_b200.ep import ExpertParallelBlock, ExpertParallelStack, expert_range
        from parity import assert_close

        res = {}
        if case in ("block", "block_bf16", "sigmoid", "chunked"):
            cfg = CFG if case != "sigmoid" else CFG_SIG
            bw = S.host_block(cfg, 41)
            T_r = 6 if case == "chunked" else 5
            x = S.host_x(41, world * T_r, cfg.hidden)
            e0, n = expert_range(cfg.num_experts, world, rank)
            blk = ExpertParallelBlock(local_block(bw, e0, n), cfg, expert_begin=e0, num_local=n, ops=OracleEpOps(),
                                      chunks=3 if case == "chunked" else None,
                                      partials="bf16" if case == "block_bf16" else "f32")
            xr = from_bits(x[rank * T_r:(rank + 1) * T_r])
            out = blk.forward(xr)
            ref, idx, w = O.block_forward(bw, x)
            rows = slice(rank * T_r, (rank + 1) * T_r)
            # every rank routes every gathered token: its packed routing covers all ranks'
            # rows, in the gathered order (with C chunks: chunk-major, then rank, then row)
            pk = blk.buffers(T_r, xr.device).packed_all.numpy().view(np.uint32)
            C = 3 if case == "chunked" else 1
            Tc = T_r // C
            order = [r * T_r + c * Tc + i for c in range(C) for r in range(world) for i in range(Tc)]
            assert np.array_equal(pk, O.pack_routing(idx, w)[order]), "routing differs"
            m = assert_close(bits(out), ref[rows], f"ep rank {rank}")
            res = {"frac_exact": m["frac_exact"]}
        elif case == "stack":
            blocks_host = [S.host_block(CFG, 50 + l) for l in range(3)]
            rng = np.random.default_rng(9)
            norms = [None] + [S.f32_to_bf16_bits(rng.uniform(0.5, 1.5, CFG.hidden).astype(np.float32))
                              for _ in range(2)]
            T_r = 4
            x = S.host_x(52, world * T_r, CFG.hidden)
            e0, n = expert_range(CFG.num_experts, world, rank)
            blocks = [ExpertParallelBlock(local_block(b, e0, n), CFG, expert_begin=e0, num_local=n,
                                          ops=OracleEpOps()) for b in blocks_host]
            stack = ExpertParallelStack(blocks, [None if w is None else from_bits(w) for w in norms])
            out = stack.forward(from_bits(x[rank * T_r:(rank + 1) * T_r]))
            ref = O.stack_forward(blocks_host, norms, x)
            m = assert_close(bits(out), ref[rank * T_r:(rank + 1) * T_r], f"ep stack rank {rank}")
            res = {"frac_exact": m["frac_exact"]}
        q.put((rank, "ok", res))
    except Exception as e:  # reported to the parent, which fails the test
        import traceback
        q.put((rank, "error", traceback.format_exc()))
    finally:
        dist.destroy_process_group()


def _run(case, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, payload = q.get(timeout=240)
            results[rank] = (status, payload)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank in range(world):
        status, payload = results[rank]
        assert status == "ok", f"rank {rank}:\n{payload}"
    return results


@pytest.mark.parametrize("world", [2, 4])
def test_ep_block_matches_single_device_oracle(world):
    """fp32 partial sums (the default): the single-device result up to the fp32
    association of the k-term sum, so nearly every element is bit-identical."""
    r = _run("block", world)
    assert all(p[1]["frac_exact"] > 0.99 for p in r.values()), r


def test_ep_block_bf16_partials_world2():
    """bf16 partial sums (partials="bf16"): within the parity tolerance of the
    single-device block (checked in every rank)."""
    _run("block_bf16", 2)


def test_ep_sigmoid_routing_world2():
    _run("sigmoid", 2)


def test_ep_chunked_overlap_world2():
    """Three token chunks per block: gathers and all-to-alls issued asynchronously so that
    they overlap the next chunk's experts; same results as the single-device block."""
    _run("chunked", 2)


def test_ep_stack_with_fused_norm_world2():
    _run("stack", 2)


def test_expert_range_and_local_weights():
    from mlx_rs_b200.ep import expert_range
    assert [expert_range(128, 8, r) for r in (0, 7)] == [(0, 16), (112, 16)]
    with pytest.raises(Exception):
        expert_range(60, 8, 0)
    with pytest.raises(Exception):
        expert_range(8, 2, 2)
