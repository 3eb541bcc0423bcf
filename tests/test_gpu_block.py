"""GPU parity of the CUDA path against the oracle (golden fixtures and live oracle runs).

Routing (index sets in order, bf16 weights, per-expert offsets and token grouping) must
match bit for bit; block outputs must meet the tolerance in tests/parity.py.
"""
import os

import numpy as np
import pytest

import mlx_rs_b200.synth as S
from parity import ULP_TOL, ULP_TOL_TC, assert_close

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _torch():
    import torch
    return torch


def _check_routing(got, idx, w, offsets, perm, name):
    _, gidx, gw, goff, gperm = got
    assert np.array_equal(gidx.reshape(idx.shape), idx), f"{name}: expert indices differ"
    assert np.array_equal(gw.reshape(w.shape), w), f"{name}: combine weights differ"
    assert np.array_equal(goff, offsets), f"{name}: per-expert offsets differ"
    assert np.array_equal(gperm, perm), f"{name}: per-expert grouping differs"


@pytest.mark.parametrize("name", ["block_qwen_shared", "block_qwen3_renorm", "block_lfm2_sigmoid",
                                  "block_lfm2_softmax_bias"])
def test_block_golden(name):
    import golden_cases as G
    from gpu_util import make_block, run_block
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    bw = G.block_from_dict(z)
    blk = make_block(bw)
    got = run_block(blk, z["x"])
    _check_routing(got, z["idx"], z["weights"], z["offsets"], z["perm"], name)
    assert_close(got[0].reshape(z["out"].shape), z["out"], name)


def test_gather_qmm_golden():
    torch = _torch()
    from mlx_rs_b200 import ops
    from gpu_util import dev_bits, to_dev
    z = np.load(os.path.join(GOLDEN, "gather_qmm.npz"))
    x, w, s, b = to_dev(z["x"]), torch.from_numpy(z["w"].view(np.int32)).cuda(), to_dev(z["s"]), to_dev(z["b"])
    T, k = z["rhs"].shape
    rhs = torch.from_numpy(z["rhs"].view(np.int32)).cuda()
    # SwitchGLU form: x [T,1,1,K] with rhs [T,k] -> [T,k,1,N]
    out = ops.gather_qmm(x.reshape(T, 1, 1, -1), w, s, b, None, rhs, True, 64, 4, False)
    assert tuple(out.shape) == (T, k, 1, w.shape[1])
    assert_close(dev_bits(out).reshape(T * k, -1), z["out"], "gather_qmm")
    lhs = torch.from_numpy(z["lhs"].view(np.int32)).cuda()
    rhs2 = torch.from_numpy(z["rhs2"].view(np.int32)).cuda()
    out2 = ops.gather_qmm(x.reshape(T, 1, -1), w, s, b, lhs, rhs2, True, 64, 4, False)
    assert_close(dev_bits(out2).reshape(len(z["lhs"]), -1), z["out_lhs"], "gather_qmm lhs")


def test_quantized_matmul_golden():
    torch = _torch()
    from mlx_rs_b200 import ops
    from gpu_util import dev_bits, to_dev
    z = np.load(os.path.join(GOLDEN, "qmm.npz"))
    out = ops.quantized_matmul(to_dev(z["x"]), torch.from_numpy(z["w"].view(np.int32)).cuda(), to_dev(z["s"]),
                               to_dev(z["b"]), True, 64, 4)
    assert_close(dev_bits(out), z["out"], "qmm")


def test_rms_norm_golden_bit_exact():
    from mlx_rs_b200 import ops
    from gpu_util import dev_bits, to_dev
    z = np.load(os.path.join(GOLDEN, "rms_norm.npz"))
    out = ops.fast_rms_norm(to_dev(z["x"]), to_dev(z["w"]), float(z["eps"][0]))
    assert np.array_equal(dev_bits(out), z["out"])


# ----------------------------------------------------------------------------------
# live oracle comparisons at the benchmark block shapes
# ----------------------------------------------------------------------------------

_BLOCKS = {}


def _block(cfg, seed, bias_std=None):
    from gpu_util import make_block
    key = (cfg, seed, bias_std)
    if key not in _BLOCKS:
        bw = S.host_block(cfg, seed, bias_std)
        _BLOCKS[key] = (bw, make_block(bw))
    return _BLOCKS[key]


def _live(cfg, seed, T, bias_std=None, x_seed=None, ulp_tol=ULP_TOL):
    import oracle as O
    from gpu_util import run_block
    bw, blk = _block(cfg, seed, bias_std)
    x = S.host_x(seed if x_seed is None else x_seed, T, cfg.hidden)
    got = run_block(blk, x)
    y, idx, w = O.block_forward(bw, x)
    off, perm = O.group_by_expert(idx, cfg.num_experts)
    name = f"{cfg.name or cfg} T={T}"
    _check_routing(got, idx, w, off, perm, name)
    return assert_close(got[0].reshape(y.shape), y, name, ulp_tol)


@pytest.mark.parametrize("T", [1, 8, 32, 64])
def test_qwen3_30b_decode(T):
    _live(S.QWEN3_30B_A3B, 1, T)


@pytest.mark.parametrize("T", [1, 24])
def test_qwen15_moe_shared_expert(T):
    _live(S.QWEN15_MOE_A27B, 0, T)


@pytest.mark.parametrize("T", [1, 17])
def test_lfm2_sigmoid_routing(T):
    _live(S.LFM2_8B_A1B, 3, T)


def test_lfm2_reference_softmax_bias_routing():
    from dataclasses import replace
    cfg = replace(S.LFM2_8B_A1B, scoring=S.SCORING_SOFTMAX_BIAS, name="lfm2-softmax-bias")
    _live(cfg, 3, 9)


def test_qwen3_skewed_routing():
    """Skewed expert loads: a per-expert logit bias ~ N(0, 2) added before the softmax."""
    from dataclasses import replace
    cfg = replace(S.QWEN3_30B_A3B, scoring=S.SCORING_SOFTMAX_BIAS, name="qwen3-skewed")
    _live(cfg, 2, 96, bias_std=2.0)


def _live_full(cfg, seed, T, bias_std=None, x_seed=None, ulp_tol=ULP_TOL_TC):
    """A prefill-sized block against the oracle on every output row (the oracle runs the
    whole batch on the host cores), routing and grouping bit-exact; the block then runs
    once more under moe_block_profile, which raises if a bounded device wait expired."""
    m = _live(cfg, seed, T, bias_std=bias_std, x_seed=x_seed, ulp_tol=ulp_tol)
    _, blk = _block(cfg, seed, bias_std)
    _profile_clean(blk, S.host_x(seed if x_seed is None else x_seed, T, cfg.hidden))
    return m


def test_prefill_qwen3_T4096_all_rows():
    """The prefill workload (Qwen3-30B-A3B block, T=4096, near-uniform routing: every
    expert on the tcgen05 GEMM): all 4096 output rows against the oracle."""
    _live_full(S.QWEN3_30B_A3B, 2, 4096)


def test_prefill_qwen3_skewed_T4096_all_rows():
    """The skewed prefill workload (per-expert logit bias ~ N(0, 2) before the softmax:
    experts from a handful of rows on the GEMV to over a thousand on uneven tcgen05
    tiles): all 4096 output rows against the oracle."""
    from dataclasses import replace
    cfg = replace(S.QWEN3_30B_A3B, scoring=S.SCORING_SOFTMAX_BIAS, name="qwen3-skewed")
    _live_full(cfg, 2, 4096, bias_std=2.0)


@pytest.mark.parametrize("cname,seed,T", [
    ("QWEN3_30B_A3B", 2, 1), ("QWEN3_30B_A3B", 2, 64), ("QWEN3_30B_A3B", 2, 65),
    ("QWEN3_30B_A3B", 2, 1001), ("QWEN3_30B_A3B", 2, 4096),
    ("QWEN15_MOE_A27B", 0, 77), ("QWEN15_MOE_A27B", 0, 203), ("QWEN15_MOE_A27B", 0, 512),
    ("LFM2_8B_A1B", 3, 1024)])
def test_router_logits_bit_exact(cname, seed, T):
    """moe_block_router_logits against the oracle's router logits (and, with a shared
    expert gate, its quantized_matmul of shared_expert_gate), bit for bit, on every
    token: the small-batch router kernels (T <= 64) and the shared-memory one (larger
    batches, including ragged last token groups)."""
    import oracle as O
    from gpu_util import dev_bits, to_dev
    cfg = getattr(S, cname)
    bw, blk = _block(cfg, seed)
    x = S.host_x(seed, T, cfg.hidden)
    got = dev_bits(blk.router_logits(to_dev(x)))
    _, _, logits, _ = O.route(bw, x)
    E = cfg.num_experts
    assert np.array_equal(got[:, :E], logits), f"{cname} T={T}: router logits differ"
    if cfg.shared_inter > 0 and cfg.has_shared_gate:
        g = bw.shared_expert_gate
        ref = O.qmm(x, g.w, g.scales, g.biases)
        assert np.array_equal(got[:, E:E + 1], ref), f"{cname} T={T}: shared_expert_gate logit differs"


def test_deterministic_and_batch_independent():
    from gpu_util import run_block
    cfg = S.QWEN3_30B_A3B
    bw, blk = _block(cfg, 1)
    x = S.host_x(5, 40, cfg.hidden)
    a = run_block(blk, x)
    b = run_block(blk, x)
    for u, v in zip(a, b):
        assert np.array_equal(u, v)
    part = run_block(blk, x[:7])
    assert np.array_equal(part[0].reshape(7, -1), a[0].reshape(40, -1)[:7])


def test_zero_tokens_and_errors():
    torch = _torch()
    from mlx_rs_b200 import MlxError, ops
    cfg = S.QWEN3_30B_A3B
    bw, blk = _block(cfg, 1)
    out = blk.forward(torch.empty(0, cfg.hidden, dtype=torch.bfloat16, device="cuda"))
    assert out.shape == (0, cfg.hidden)
    x = torch.zeros(2, 256, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(64, 256 * 3 // 32, dtype=torch.int32, device="cuda")
    s = torch.zeros(64, 256 // 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(MlxError) as e:
        ops.quantized_matmul(x, w, s, s, True, 64, 3)
    assert "rc=2" in str(e.value) and "mlx_quantized_matmul" in str(e.value)
    with pytest.raises(MlxError):
        ops.quantized_matmul(x, w, s, s, False, 64, 4)


def test_stack_layers_match_oracle():
    """Three Qwen3-shaped blocks with RMSNorm between them (the layer structure of the
    expert-parallel stack), T=16, compared layer by layer: each GPU block and norm gets
    the oracle's input of that layer (a last-bit difference in one layer's output may
    legitimately change the next layer's routing, so the layers are checked separately);
    the full GPU stack then runs end to end."""
    torch = _torch()
    import oracle as O
    from mlx_rs_b200.block import MoeStack, RmsNorm
    from gpu_util import dev_bits, make_block, to_dev
    cfg = S.QWEN3_30B_A3B
    bws = [S.host_block(cfg, 100 + l) for l in range(3)]
    rng = np.random.default_rng(9)
    norms = [S.f32_to_bf16_bits(rng.uniform(0.5, 1.5, cfg.hidden).astype(np.float32)) for _ in range(3)]
    x = S.host_x(4, 16, cfg.hidden)
    blocks = [make_block(b) for b in bws]
    rms = [RmsNorm(to_dev(n), 1e-6) for n in norms]
    h = x
    for l in range(3):
        if l > 0:
            hn = O.rms_norm(h, norms[l], 1e-6)
            got = dev_bits(rms[l](to_dev(h)))
            assert np.array_equal(got, hn), f"rms_norm layer {l}"
            h = hn
        y, _, _ = O.block_forward(bws[l], h)
        assert_close(dev_bits(blocks[l](to_dev(h))).reshape(y.shape), y, f"layer {l}")
        h = y
    out = MoeStack(blocks, rms)(to_dev(x))
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()


# ----------------------------------------------------------------------------------
# tensor-core (tcgen05) prefill path
# ----------------------------------------------------------------------------------

def _profile_clean(blk, x_bits):
    """Runs moe_block_profile, which raises if a bounded device wait expired."""
    from gpu_util import to_dev
    _, stages, _ = blk.profile(to_dev(x_bits))
    return stages


def test_tc_prefill_qwen15_shared_T512():
    """Qwen1.5-MoE shape at T=512: routed experts (~34 rows each) and the shared expert
    both take the tcgen05 GEMM; every row compared with the oracle."""
    _live(S.QWEN15_MOE_A27B, 0, 512, x_seed=50, ulp_tol=ULP_TOL_TC)
    bw, blk = _block(S.QWEN15_MOE_A27B, 0)
    _profile_clean(blk, S.host_x(51, 512, 2048))


def test_tc_prefill_lfm2_T1024_all_rows():
    """LFM2-8B-A1B block (sigmoid + bias selection) at T=1024: all rows against the oracle."""
    _live_full(S.LFM2_8B_A1B, 3, 1024)


@pytest.mark.parametrize("T", [3, 40])
def test_tc_forced_small_tiles(T, monkeypatch):
    """The tcgen05 path forced on decode-sized inputs (tiles of 1..16 rows, N=16)."""
    monkeypatch.setenv("MOE_B200_TC", "1")
    _live(S.QWEN3_30B_A3B, 1, T, x_seed=60 + T, ulp_tol=ULP_TOL_TC)
    _, blk = _block(S.QWEN3_30B_A3B, 1)
    _profile_clean(blk, S.host_x(61, T, 2048))


def test_tc_and_gemv_paths_agree(monkeypatch):
    """Same block, same tokens: the tcgen05 path (bf16-rounded dequantised weights) and the
    GEMV path (fp32 scale folding) agree within the parity tolerance."""
    from gpu_util import run_block
    _, blk = _block(S.QWEN3_30B_A3B, 1)
    x = S.host_x(70, 200, 2048)
    monkeypatch.setenv("MOE_B200_TC", "1")
    a = run_block(blk, x)
    monkeypatch.setenv("MOE_B200_TC", "0")
    b = run_block(blk, x)
    for u, v in zip(a[1:], b[1:]):
        assert np.array_equal(u, v)
    assert_close(a[0].reshape(200, -1), b[0].reshape(200, -1), "tc vs gemv", ULP_TOL_TC)


# ----------------------------------------------------------------------------------
# fused routing (router + top-k + grouping in one launch, decode-sized batches)
# ----------------------------------------------------------------------------------

@pytest.mark.parametrize("cfg_name,seed", [("QWEN3_30B_A3B", 1), ("QWEN15_MOE_A27B", 0), ("LFM2_8B_A1B", 3)])
def test_fused_routing_matches_three_launches(cfg_name, seed, monkeypatch):
    """Decode-sized batches route through one fused launch whose last CTAs run top-k and
    the grouping; its results equal the three-launch path bit for bit, on repeated calls
    (the ticket counters return to zero) and for every batch size up to the limit."""
    from gpu_util import run_block
    cfg = getattr(S, cfg_name)
    _, blk = _block(cfg, seed)
    for T in (1, 3, 4, 5, 17, 63, 64):
        x = S.host_x(500 + T, T, cfg.hidden)
        monkeypatch.setenv("MOE_B200_FUSED_ROUTE", "0")
        ref = run_block(blk, x)
        monkeypatch.setenv("MOE_B200_FUSED_ROUTE", "1")
        for _ in range(2):
            got = run_block(blk, x)
            for u, v in zip(got[1:], ref[1:]):
                assert np.array_equal(u, v), (cfg_name, T)
            assert np.array_equal(got[0], ref[0]), (cfg_name, T)


@pytest.mark.parametrize("cfg_name,seed,T", [("QWEN15_MOE_A27B", 0, 1), ("QWEN3_30B_A3B", 1, 2),
                                             ("LFM2_8B_A1B", 3, 1)])
def test_split_k_gemv_matches_unsplit_and_oracle(cfg_name, seed, T, monkeypatch):
    """Few-token GEMVs (the shared expert, T <= 2 routed experts) split K over more CTAs
    and add the fp32 partials in split order; within tolerance of the unsplit GEMV and of
    the oracle, routing unchanged."""
    import oracle as O
    from gpu_util import run_block
    cfg = getattr(S, cfg_name)
    bw, blk = _block(cfg, seed)
    x = S.host_x(600 + T, T, cfg.hidden)
    monkeypatch.setenv("MOE_B200_SPLITK", "0")
    ref = run_block(blk, x)
    monkeypatch.setenv("MOE_B200_SPLITK", "1")
    got = run_block(blk, x)
    for u, v in zip(got[1:], ref[1:]):
        assert np.array_equal(u, v)
    assert_close(got[0].reshape(T, -1), ref[0].reshape(T, -1), f"{cfg_name} split vs unsplit", ULP_TOL)
    y, _, _ = O.block_forward(bw, x)
    assert_close(got[0].reshape(T, -1), y, f"{cfg_name} split vs oracle", ULP_TOL)


@pytest.mark.parametrize("cfg_name,seed,T", [("QWEN3_30B_A3B", 1, 64), ("LFM2_8B_A1B", 3, 32),
                                              ("QWEN15_MOE_A27B", 2, 48)])
def test_whole_k_scale_gemv_bit_identical(cfg_name, seed, T, monkeypatch):
    """The decode GEMV with each unit's scales for all of K copied once (16-warp CTAs)
    computes exactly what the per-chunk scale copies compute: same bits, and the oracle
    within tolerance."""
    import oracle as O
    from gpu_util import run_block
    cfg = getattr(S, cfg_name)
    bw, blk = _block(cfg, seed)
    x = S.host_x(700 + T, T, cfg.hidden)
    monkeypatch.setenv("MOE_B200_GEMV_FK", "0")
    ref = run_block(blk, x)
    monkeypatch.setenv("MOE_B200_GEMV_FK", "1")
    got = run_block(blk, x)
    for u, v in zip(got, ref):
        assert np.array_equal(u, v)
    y, _, _ = O.block_forward(bw, x)
    assert_close(got[0].reshape(T, -1), y, f"{cfg_name} whole-K scales vs oracle", ULP_TOL)


# ----------------------------------------------------------------------------------
# the decoder layer's FFN half: x + block(RmsNorm(x)), residual fused into the combine
# ----------------------------------------------------------------------------------

@pytest.mark.parametrize("cfg_name,seed,T", [("QWEN3_30B_A3B", 1, 64), ("QWEN15_MOE_A27B", 2, 24),
                                              ("LFM2_8B_A1B", 3, 512)])
def test_layer_ffn_matches_oracle_and_unfused(cfg_name, seed, T):
    """Normed rows bit-exact with the oracle's RMSNorm, routing bit-exact on them, the
    fused residual bit-identical to block output + x added in bf16, and within tolerance
    of the oracle layer."""
    torch = _torch()
    import oracle as O
    from gpu_util import dev_bits, to_dev
    cfg = getattr(S, cfg_name)
    bw, blk = _block(cfg, seed)
    x_bits = S.host_x(800 + T, T, cfg.hidden)
    nw_bits = S.f32_to_bf16_bits(np.random.default_rng(seed).uniform(0.5, 1.5, cfg.hidden).astype(np.float32))
    x, nw = to_dev(x_bits), to_dev(nw_bits)
    normed = torch.empty_like(x)
    out = blk.forward_layer(x, nw, 1e-6, normed=normed)
    unfused = blk.forward(normed) + x
    idx, w, _, _ = blk.route(normed)
    torch.cuda.synchronize()
    y, h_ref, idx_ref, w_ref = O.layer_ffn_forward(bw, x_bits, nw_bits, 1e-6)
    assert np.array_equal(dev_bits(normed), h_ref), "RMSNorm differs"
    assert np.array_equal(dev_bits(idx).reshape(idx_ref.shape), idx_ref), "routing differs"
    assert np.array_equal(dev_bits(w).reshape(w_ref.shape), w_ref), "combine weights differ"
    assert np.array_equal(dev_bits(out), dev_bits(unfused)), "fused residual differs from block + x"
    tol = ULP_TOL_TC if T >= 512 else ULP_TOL
    assert_close(dev_bits(out).reshape(y.shape), y, f"{cfg_name} layer vs oracle", tol)


def test_residual_stack_and_layer_errors():
    """Layer by layer against the oracle (each layer fed the oracle's input: a last-bit
    difference in one layer can flip a later layer's top-k choice, so the stack is not
    compared end to end), and the stack equals its layers applied in turn, bit for bit."""
    torch = _torch()
    import oracle as O
    from mlx_rs_b200._lib import MlxError
    from mlx_rs_b200.block import MoeStack, RmsNorm
    from gpu_util import dev_bits, make_block, to_dev
    cfg = S.QWEN3_30B_A3B
    bws = [S.host_block(cfg, 110 + l) for l in range(3)]
    rng = np.random.default_rng(11)
    norms = [S.f32_to_bf16_bits(rng.uniform(0.5, 1.5, cfg.hidden).astype(np.float32)) for _ in range(3)]
    x = S.host_x(12, 32, cfg.hidden)
    blocks = [make_block(b) for b in bws]
    h = x
    for l in range(3):
        y, _, _, _ = O.layer_ffn_forward(bws[l], h, norms[l], 1e-6)
        got = dev_bits(blocks[l].forward_layer(to_dev(h), to_dev(norms[l]), 1e-6))
        assert_close(got.reshape(y.shape), y, f"layer {l} vs oracle", ULP_TOL)
        h = y
    stack = MoeStack(blocks, [RmsNorm(to_dev(n), 1e-6) for n in norms], residual=True)
    xd = to_dev(x)
    out = dev_bits(stack(xd))
    hd = xd
    for l in range(3):
        hd = blocks[l].forward_layer(hd, to_dev(norms[l]), 1e-6)
    assert np.array_equal(out, dev_bits(hd))
    with pytest.raises(MlxError):
        blocks[0].forward_layer(xd, to_dev(norms[0]), 1e-6, out=xd)  # out aliases x
    torch.cuda.synchronize()


def test_graphed_residual_stack_bit_identical_to_eager():
    """A 3-layer residual stack captured once and replayed per step: each replay's output
    is bit-identical to the eager stack on the same input."""
    torch = _torch()
    from mlx_rs_b200.block import MoeStack, RmsNorm
    from mlx_rs_b200.graph import GraphedForward
    from gpu_util import dev_bits, make_block, to_dev
    cfg = S.QWEN3_30B_A3B
    bws = [S.host_block(cfg, 120 + l) for l in range(3)]
    norms = [RmsNorm(to_dev(S.f32_to_bf16_bits(np.full(cfg.hidden, 1.0 + 0.1 * l, np.float32))), 1e-6)
             for l in range(3)]
    stack = MoeStack([make_block(b) for b in bws], norms, residual=True)
    xs = [to_dev(S.host_x(130 + i, 8, cfg.hidden)) for i in range(3)]
    g = GraphedForward(stack, xs[0])
    for x in xs:
        want = dev_bits(stack(x))
        got = dev_bits(g(x))
        assert np.array_equal(got, want)
    torch.cuda.synchronize()


@pytest.mark.parametrize("cfg,T", [
    (S.MoeConfig(256, 512, 32, 128, 0, S.SCORING_SOFTMAX, True, False, name="max-experts-topk"), 17),
    (S.MoeConfig(256, 512, 32, 128, 0, S.SCORING_SOFTMAX, False, False, name="max-experts-topk"), 1),
    (S.MoeConfig(256, 1, 1, 128, 0, S.SCORING_SOFTMAX, False, False, name="one-expert"), 9),
    (S.MoeConfig(256, 3, 2, 128, 0, S.SCORING_SIGMOID_BIAS_SELECT, True, False, name="three-experts"), 13),
])
def test_extreme_shapes_match_oracle(cfg, T):
    """The ABI's limits (512 experts, top-32) and the smallest expert sets: routing and
    grouping bit-exact, outputs within tolerance."""
    _live(cfg, 31, T)


@pytest.mark.parametrize("cfg,T", [
    # I % 128 != 0: gate/up on the GEMV for every expert, down hybrid (tcgen05 from 32 rows)
    (S.MoeConfig(256, 8, 2, 192, 0, S.SCORING_SOFTMAX_BIAS, True, False, name="gemv-gate-up-hybrid-down"), 80),
    # H % 128 != 0: gate/up hybrid, down on the GEMV for every expert
    (S.MoeConfig(192, 8, 2, 128, 0, S.SCORING_SOFTMAX_BIAS, True, False, name="hybrid-gate-up-gemv-down"), 80),
])
def test_hybrid_with_one_projection_on_one_kernel(cfg, T):
    """Hybrid steps where only one projection's shape suits the tensor-core kernel: the
    other projection reads rows of every expert, so the two kernels' chains must not run
    on separate streams; outputs against the oracle, routing bit-exact. Skewed routing
    (per-expert selection bias) gives some experts 32 rows or more while the rows stay
    under 24 per expert on average, so both kernels run (the tensor-core tolerance)."""
    import oracle as O
    bw, _ = _block(cfg, 41, 1.0)
    idx = O.block_forward(bw, S.host_x(41, T, cfg.hidden))[1]
    cnt = np.bincount(idx.ravel(), minlength=cfg.num_experts)
    assert cnt.max() >= 32 and cnt.min() < 32 and idx.size < 24 * cfg.num_experts
    _live(cfg, 41, T, bias_std=1.0, ulp_tol=ULP_TOL_TC)


@pytest.mark.parametrize("cfg_name,seed,T", [("QWEN3_30B_A3B", 1, 64), ("LFM2_8B_A1B", 3, 32)])
def test_int8_gemv_path_matches_oracle(cfg_name, seed, T, monkeypatch):
    """The opt-in integer decode GEMV (u8 weights, two s8 limbs of each token row, int32
    MMA): routing unchanged, outputs within the parity tolerance of the oracle."""
    import oracle as O
    from gpu_util import run_block
    cfg = getattr(S, cfg_name)
    bw, blk = _block(cfg, seed)
    x = S.host_x(900 + T, T, cfg.hidden)
    monkeypatch.setenv("MOE_B200_GEMV_I8", "0")
    ref = run_block(blk, x)
    monkeypatch.setenv("MOE_B200_GEMV_I8", "1")
    got = run_block(blk, x)
    y, idx, w = O.block_forward(bw, x)
    assert np.array_equal(got[1].reshape(idx.shape), idx)
    assert np.array_equal(got[2].reshape(w.shape), w)
    assert_close(got[0].reshape(T, -1), y, f"{cfg_name} int8 GEMV vs oracle", ULP_TOL)
    # the integer kernel really ran: its fixed-point token rows round differently from the
    # bf16 kernel's, so the two outputs are not bit-identical
    assert not np.array_equal(got[0], ref[0]), "MOE_B200_GEMV_I8=1 did not reach the integer kernel"


def test_int8_gemv_propagates_non_finite_tokens(monkeypatch):
    """A token row holding inf: the integer kernel writes NaN for that token's outputs (as
    the bf16 kernel's arithmetic does: inf times weights of both signs), other tokens stay
    finite and within tolerance of the bf16 kernel."""
    torch = _torch()
    from gpu_util import dev_bits, to_dev
    cfg = S.QWEN3_30B_A3B
    bw, blk = _block(cfg, 1)
    x = S.host_x(950, 64, cfg.hidden).copy()
    x[5, 100] = 0x7F80  # +inf
    monkeypatch.setenv("MOE_B200_GEMV_I8", "1")
    out = blk.forward(to_dev(x))
    torch.cuda.synchronize()
    y = out.float().cpu().numpy()
    assert not np.isfinite(y[5]).any()
    assert np.isfinite(np.delete(y, 5, axis=0)).all()
    monkeypatch.setenv("MOE_B200_GEMV_I8", "0")
    ref = dev_bits(blk.forward(to_dev(x)))
    keep = [t for t in range(64) if t != 5]
    assert_close(dev_bits(out)[keep], ref[keep], "int8 vs bf16 kernel, finite tokens", ULP_TOL)


# ----------------------------------------------------------------------------------
# op-level drop-ins on the tensor-core branch, graph replays against the oracle
# ----------------------------------------------------------------------------------

def test_gather_qmm_hybrid_tc_and_gemv_vs_oracle():
    """ops.gather_qmm in the SwitchGLU form at Qwen3-30B-A3B shapes with 512 tokens (4096
    rows over 128 experts, ~32 each): experts with 32 rows or more run on the tcgen05 GEMM,
    the others on the GEMV, in one call; every row against the oracle, both the gate/up
    form (x [T,1,1,H], rhs [T,k]) and the down form (x [T,k,1,I])."""
    torch = _torch()
    import oracle as O
    from mlx_rs_b200 import ops
    from gpu_util import dev_bits, to_dev
    cfg = S.QWEN3_30B_A3B
    bw, _ = _block(cfg, 1)
    T, k = 512, cfg.top_k
    x = S.host_x(1200, T, cfg.hidden)
    idx, _, _, _ = O.route(bw, x)
    rhs = torch.from_numpy(idx.view(np.int32)).cuda()
    wg = torch.from_numpy(bw.gate.w.view(np.int32)).cuda()
    sg, bg = to_dev(bw.gate.scales), to_dev(bw.gate.biases)
    out = ops.gather_qmm(to_dev(x).reshape(T, 1, 1, -1), wg, sg, bg, None, rhs, True, 64, 4, False)
    assert tuple(out.shape) == (T, k, 1, cfg.moe_inter)
    want = O.gather_qmm(x, bw.gate.w, bw.gate.scales, bw.gate.biases, idx, x_repeat=k)
    assert_close(dev_bits(out).reshape(T * k, -1), want, "gather_qmm gate/up form", ULP_TOL_TC)
    h = S.f32_to_bf16_bits(np.random.default_rng(3).standard_normal((T * k, cfg.moe_inter)).astype(np.float32))
    wd = torch.from_numpy(bw.down.w.view(np.int32)).cuda()
    out = ops.gather_qmm(to_dev(h).reshape(T, k, 1, -1), wd, to_dev(bw.down.scales), to_dev(bw.down.biases),
                         None, rhs, True, 64, 4, False)
    want = O.gather_qmm(h, bw.down.w, bw.down.scales, bw.down.biases, idx, x_repeat=1)
    assert_close(dev_bits(out).reshape(T * k, -1), want, "gather_qmm down form", ULP_TOL_TC)


@pytest.mark.parametrize("M", [7, 256, 1000])
def test_quantized_matmul_gemv_and_tc_vs_oracle(M):
    """quantized_matmul at the shared expert's shape: M < 32 on the GEMV, more rows on the
    tcgen05 GEMM (token tiles in order, a ragged last tile at M=1000)."""
    torch = _torch()
    import oracle as O
    from mlx_rs_b200 import ops
    from gpu_util import dev_bits, to_dev
    bw, _ = _block(S.QWEN15_MOE_A27B, 0)
    q = bw.shared_gate
    x = S.host_x(1300 + M, M, 2048)
    out = ops.quantized_matmul(to_dev(x), torch.from_numpy(q.w.view(np.int32)).cuda(), to_dev(q.scales),
                               to_dev(q.biases), True, 64, 4)
    want = O.qmm(x, q.w, q.scales, q.biases)
    assert_close(dev_bits(out), want, f"qmm M={M}", ULP_TOL_TC if M >= 32 else ULP_TOL)


@pytest.mark.parametrize("cfg_name,seed,T", [("QWEN3_30B_A3B", 1, 1), ("QWEN3_30B_A3B", 1, 64),
                                              ("QWEN15_MOE_A27B", 0, 1), ("LFM2_8B_A1B", 3, 8)])
def test_graphed_block_and_layer_replays_vs_oracle(cfg_name, seed, T):
    """The decode step as the serving loop runs it: a block and a decoder layer's FFN half
    each captured once (graph.GraphedForward) and replayed on new tokens every step; every
    replay is compared with the oracle (routing of the block bit-exact through the same
    captured buffers, outputs within tolerance)."""
    torch = _torch()
    import oracle as O
    from mlx_rs_b200.graph import GraphedForward
    from gpu_util import dev_bits, to_dev
    cfg = getattr(S, cfg_name)
    bw, blk = _block(cfg, seed)
    nw = S.f32_to_bf16_bits(np.random.default_rng(seed + 7).uniform(0.5, 1.5, cfg.hidden).astype(np.float32))
    nwd = to_dev(nw)
    xs = [S.host_x(1400 + 10 * T + i, T, cfg.hidden) for i in range(3)]
    gb = GraphedForward(lambda xd: blk.forward(xd), to_dev(xs[0]))
    gl = GraphedForward(lambda xd: blk.forward_layer(xd, nwd, 1e-6), to_dev(xs[0]))
    for i, x in enumerate(xs):
        got = dev_bits(gb(to_dev(x)))
        y, _, _ = O.block_forward(bw, x)
        assert_close(got.reshape(y.shape), y, f"{cfg_name} T={T} graphed block replay {i}")
        got = dev_bits(gl(to_dev(x)))
        yl, _, _, _ = O.layer_ffn_forward(bw, x, nw, 1e-6)
        assert_close(got.reshape(yl.shape), yl, f"{cfg_name} T={T} graphed layer replay {i}")
    torch.cuda.synchronize()


# ----------------------------------------------------------------------------------
# the fused decode kernel (T <= 8: the whole block in one cooperative launch)
# ----------------------------------------------------------------------------------

@pytest.mark.parametrize("cfg_name,seed", [("QWEN3_30B_A3B", 1), ("QWEN15_MOE_A27B", 0), ("LFM2_8B_A1B", 3)])
def test_decode_kernel_matches_launch_chain_and_oracle(cfg_name, seed, monkeypatch):
    """For every T up to 8: the one-launch decode kernel against the oracle (routing of
    the launch chain bit-exact, outputs within tolerance) and against the launch chain
    (MOE_B200_DECODE=0), on repeated calls (the grid barrier word is reused without a
    reset); moe_block_profile reports no expired wait."""
    import oracle as O
    from gpu_util import run_block, to_dev
    cfg = getattr(S, cfg_name)
    bw, blk = _block(cfg, seed)
    for T in (1, 2, 3, 5, 8):
        x = S.host_x(1500 + T, T, cfg.hidden)
        monkeypatch.setenv("MOE_B200_DECODE", "0")
        ref = run_block(blk, x)
        monkeypatch.setenv("MOE_B200_DECODE", "1")
        got = run_block(blk, x)
        again = run_block(blk, x)
        assert np.array_equal(got[0], again[0]), (cfg_name, T)
        y, idx, w = O.block_forward(bw, x)
        assert np.array_equal(got[1].reshape(idx.shape), idx)
        assert_close(got[0].reshape(T, -1), y, f"{cfg_name} T={T} decode kernel vs oracle")
        assert_close(got[0].reshape(T, -1), ref[0].reshape(T, -1), f"{cfg_name} T={T} decode kernel vs chain")
        _, st, _ = blk.profile(to_dev(x))
        assert st["gate_up"] > 0


def test_decode_kernel_layer_step_vs_oracle(monkeypatch):
    """The decoder layer's FFN half at T=4 (RMSNorm, then the decode kernel with the
    residual added in its combine) against the oracle layer."""
    monkeypatch.setenv("MOE_B200_DECODE", "1")
    torch = _torch()
    import oracle as O
    from gpu_util import dev_bits, to_dev
    cfg = S.QWEN15_MOE_A27B
    bw, blk = _block(cfg, 0)
    x = S.host_x(1600, 4, cfg.hidden)
    nw = S.f32_to_bf16_bits(np.random.default_rng(4).uniform(0.5, 1.5, cfg.hidden).astype(np.float32))
    out = blk.forward_layer(to_dev(x), to_dev(nw), 1e-6)
    torch.cuda.synchronize()
    y, _, _, _ = O.layer_ffn_forward(bw, x, nw, 1e-6)
    assert_close(dev_bits(out).reshape(y.shape), y, "decode kernel layer step")


# ----------------------------------------------------------------------------------
# the Gemma4 MoE variant (gemma4.rs Router + GELU SwitchGlu, f32 router and output)
# ----------------------------------------------------------------------------------

@pytest.mark.parametrize("T", [1, 8, 64, 512, 2048])
def test_gemma4_block_vs_oracle(T):
    """moe_gemma4_block_forward against the oracle's restatement of the reference:
    experts and f32 combine weights bit for bit (the router runs the canonical order on
    the f32 router input, softmax and renormalisation in the same IEEE operations), the
    f32 block output within the tolerance (the kernels round the GELU hidden and the
    expert outputs to bf16; at T >= 512 most experts take the tcgen05 GEMM)."""
    torch = _torch()
    import oracle as O
    from mlx_rs_b200.block import Gemma4MoeBlock
    from gpu_util import to_dev
    from parity import assert_close_f32
    cfg = S.GEMMA4_STYLE
    key = ("gemma4", cfg)
    if key not in _BLOCKS:
        bw = S.host_block(cfg, 7)
        rs, pes = S.host_gemma4_scales(cfg, 7)
        _BLOCKS[key] = (bw, rs, pes, Gemma4MoeBlock(S.to_device(bw, "cuda"), to_dev(rs), to_dev(pes)))
    bw, rs, pes, blk = _BLOCKS[key]
    x = S.host_x(1700 + T, T, cfg.hidden)
    out, idx, w = blk.forward(to_dev(x), routing=True)
    torch.cuda.synchronize()
    y, ridx, rw = O.gemma4_block_forward(bw, rs, pes, x)
    assert np.array_equal(idx.cpu().numpy().view(np.uint32), ridx), "experts differ"
    assert np.array_equal(w.cpu().numpy().view(np.uint32), rw.view(np.uint32)), "combine weights differ"
    assert out.dtype == torch.float32
    assert_close_f32(out.cpu().numpy(), y, f"gemma4 T={T}")
