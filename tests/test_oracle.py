"""CPU tests of the oracle: its numerics, its tie rule against the reference's own host
selector, and agreement with an independent numpy restatement and the golden fixtures."""
import os

import numpy as np
import pytest

import oracle as O
import mlx_rs_b200.synth as S
import numpy_ref as R
from parity import assert_close, metrics

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_exp_accuracy():
    xs = np.concatenate([np.linspace(-87, 88, 20001, dtype=np.float32),
                         np.random.default_rng(0).uniform(-20, 5, 5000).astype(np.float32)])
    got = np.array([O.exp(float(v)) for v in xs], dtype=np.float64)
    ref = np.exp(xs.astype(np.float64))
    ulp = np.spacing(ref.astype(np.float32)).astype(np.float64)
    err = np.abs(got - ref) / ulp
    assert err.max() <= 2.0, err.max()
    assert O.exp(-100.0) == 0.0
    assert O.exp(100.0) == float("inf")
    assert O.exp(0.0) == 1.0


def test_sigmoid_accuracy():
    xs = np.linspace(-30, 30, 4001, dtype=np.float32)
    got = np.array([O.sigmoid(float(v)) for v in xs])
    ref = 1 / (1 + np.exp(-xs.astype(np.float64)))
    assert np.max(np.abs(got - ref) / np.maximum(ref, 1e-30)) < 1e-6


def test_bf16_rounding_matches_numpy_helper():
    rng = np.random.default_rng(1)
    v = (rng.standard_normal(2000) * 10 ** rng.uniform(-5, 5, 2000)).astype(np.float32)
    v[:4] = [0.0, -0.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8]  # ties to even
    a = np.array([O.lib().oracle_f32_to_bf16(float(x)) for x in v], dtype=np.uint16)
    b = S.f32_to_bf16_bits(v)
    assert np.array_equal(a, b)


@pytest.mark.parametrize("K", [64, 128, 1024, 2048, 4096])
def test_canonical_dot_fast_path_is_the_definition(K):
    rng = np.random.default_rng(K)
    x = S.f32_to_bf16_bits(rng.standard_normal((3, K), dtype=np.float32))
    q = S._qweight(rng, 5, K, 64, 4)
    fast = O.qmm(x, q.w, q.scales, q.biases)
    for m in range(3):
        for n in range(5):
            d = O.dot_canonical(x[m], q.w[n], q.scales[n], q.biases[n])
            assert fast[m, n] == S.f32_to_bf16_bits(np.float32(d))


def test_qmm_against_float64():
    rng = np.random.default_rng(2)
    K, N, M = 2048, 96, 7
    x = S.f32_to_bf16_bits(rng.standard_normal((M, K), dtype=np.float32))
    q = S._qweight(rng, N, K, 64, 4)
    got = O.qmm(x, q.w, q.scales, q.biases)
    ref = S.f32_to_bf16_bits(R.qmm(R.f(x), q).astype(np.float32))
    m = metrics(got, ref)
    assert m["max_ulp"] <= 1.0 and m["frac_exact"] > 0.98, m


def test_qmm_thread_count_invariant():
    rng = np.random.default_rng(3)
    x = S.f32_to_bf16_bits(rng.standard_normal((5, 512), dtype=np.float32))
    q = S._qweight(rng, 64, 512, 64, 4)
    a = O.qmm(x, q.w, q.scales, q.biases, nthreads=1)
    b = O.qmm(x, q.w, q.scales, q.biases, nthreads=7)
    assert np.array_equal(a, b)


def test_gather_qmm_matches_qmm_per_expert():
    rng = np.random.default_rng(4)
    E, N, K, T, k = 6, 64, 256, 9, 3
    q = S._qweight(rng, E * N, K, 64, 4)
    qs = S._stack(q, E, N)
    x = S.f32_to_bf16_bits(rng.standard_normal((T, K), dtype=np.float32))
    idx = rng.integers(0, E, size=(T, k)).astype(np.uint32)
    got = O.gather_qmm(x, qs.w, qs.scales, qs.biases, idx, x_repeat=k).reshape(T, k, N)
    for t in range(T):
        for j in range(k):
            e = idx[t, j]
            ref = O.qmm(x[t:t + 1], qs.w[e], qs.scales[e], qs.biases[e])[0]
            assert np.array_equal(got[t, j], ref)
    lhs = rng.integers(0, T, size=5).astype(np.uint32)
    rhs = rng.integers(0, E, size=5).astype(np.uint32)
    g2 = O.gather_qmm(x, qs.w, qs.scales, qs.biases, rhs, lhs=lhs)
    for i in range(5):
        assert np.array_equal(g2[i], O.qmm(x[lhs[i]:lhs[i] + 1], qs.w[rhs[i]], qs.scales[rhs[i]], qs.biases[rhs[i]])[0])


def test_topk_tie_rule_matches_reference_selector():
    """The oracle's top-k equals the reference's host selector select_top_k
    (value desc, index asc) on rows full of ties."""
    rng = np.random.default_rng(5)
    levels = np.array([0.5, 0.25, 0.125, 0.0625, 0.03125, 0.0], np.float32)
    for trial in range(300):
        E = int(rng.integers(4, 130))
        k = int(rng.integers(1, min(E, 9) + 1))
        bits = S.f32_to_bf16_bits(rng.choice(levels, size=E))
        got = O.topk_rows(bits[None, :], k)[0]
        ref = [i for i, _ in R.select_top_k(list(S.bf16_bits_to_f32(bits)), k)]
        assert list(got) == ref


def test_route_topk_matches_reference_selector_on_real_router():
    cfg = S.MoeConfig(256, 64, 8, 64, 0, S.SCORING_SOFTMAX, True, False)
    bw = S.host_block(cfg, 11)
    x = S.host_x(11, 50, 256)
    idx, w, logits, probs = O.route(bw, x)
    for t in range(50):
        sel = [i for i, _ in R.select_top_k(list(S.bf16_bits_to_f32(probs[t])), 8)]
        assert list(idx[t]) == sel
    # softmax of the oracle's own logits, restated in float64, rounds to the same bf16 probs
    pr = S.f32_to_bf16_bits(R.softmax_bf(R.f(logits)).astype(np.float32))
    assert np.mean(pr == probs) > 0.99


def test_group_by_expert_is_stable():
    rng = np.random.default_rng(6)
    T, k, E = 40, 4, 10
    idx = np.stack([rng.choice(E, size=k, replace=False) for _ in range(T)]).astype(np.uint32)
    off, perm = O.group_by_expert(idx, E)
    flat = idx.reshape(-1)
    exp_perm = np.argsort(flat, kind="stable")
    assert np.array_equal(perm, exp_perm.astype(np.uint32))
    assert np.array_equal(off, np.concatenate([[0], np.cumsum(np.bincount(flat, minlength=E))]).astype(np.int32))


def test_rms_norm_against_float64():
    rng = np.random.default_rng(7)
    x = S.f32_to_bf16_bits(rng.standard_normal((16, 2048), dtype=np.float32) * 30)
    w = S.f32_to_bf16_bits(rng.uniform(0.5, 1.5, 2048).astype(np.float32))
    got = O.rms_norm(x, w, 1e-6)
    xf = R.f(x)
    r = 1 / np.sqrt(np.mean(xf * xf, axis=1, keepdims=True) + 1e-6)
    ref = S.f32_to_bf16_bits(R.bf(R.bf(xf * r) * R.f(w)).astype(np.float32))
    assert metrics(got, ref)["max_ulp"] <= 1.0


@pytest.mark.parametrize("name,cfg,T", [
    ("qwen_shared", S.MoeConfig(256, 12, 4, 128, 192, S.SCORING_SOFTMAX, False, True), 6),
    ("qwen3_renorm", S.MoeConfig(256, 16, 8, 64, 0, S.SCORING_SOFTMAX, True, False), 5),
    ("lfm2_sigmoid", S.MoeConfig(128, 8, 2, 128, 0, S.SCORING_SIGMOID_BIAS_SELECT, True, False), 7),
    ("lfm2_softmax_bias", S.MoeConfig(128, 8, 2, 64, 0, S.SCORING_SOFTMAX_BIAS, False, False), 4),
    ("max_experts_topk", S.MoeConfig(128, 512, 32, 64, 0, S.SCORING_SOFTMAX, True, False), 3),
    ("one_expert", S.MoeConfig(128, 1, 1, 64, 0, S.SCORING_SOFTMAX, False, False), 3),
    ("three_experts_sigmoid", S.MoeConfig(128, 3, 2, 64, 0, S.SCORING_SIGMOID_BIAS_SELECT, True, False), 4),
])
def test_block_oracle_vs_numpy_restatement(name, cfg, T):
    bw = S.host_block(cfg, 21)
    x = S.host_x(21, T, cfg.hidden)
    out, idx, w = O.block_forward(bw, x)
    rout, ridx, rw = R.block_forward(bw, x)
    assert np.array_equal(idx, ridx), name
    assert metrics(w, S.f32_to_bf16_bits(rw.astype(np.float32)))["max_ulp"] <= 1.0
    assert_close(out, S.f32_to_bf16_bits(rout.astype(np.float32)), name)


def test_golden_fixtures_reproduce():
    files = sorted(f for f in os.listdir(GOLDEN) if f.endswith(".npz"))
    assert files, "no golden fixtures"
    import golden_cases
    for fn in files:
        z = np.load(os.path.join(GOLDEN, fn))
        golden_cases.check_oracle_against_fixture(fn[:-4], z)


def test_layer_ffn_oracle_is_norm_block_residual():
    """x + block(rms_norm(x)): the add of two bf16 values in fp32, rounded to bf16."""
    cfg = S.MoeConfig(256, 8, 2, 128, 0, S.SCORING_SOFTMAX, True, False)
    bw = S.host_block(cfg, 5)
    x = S.host_x(6, 5, 256)
    nw = S.f32_to_bf16_bits(np.linspace(0.5, 1.5, 256, dtype=np.float32))
    out, h, idx, w = O.layer_ffn_forward(bw, x, nw, 1e-6)
    assert np.array_equal(h, O.rms_norm(x, nw, 1e-6))
    y, idx2, w2 = O.block_forward(bw, h)
    assert np.array_equal(idx, idx2) and np.array_equal(w, w2)
    assert np.array_equal(out, S.f32_to_bf16_bits(S.bf16_bits_to_f32(x) + S.bf16_bits_to_f32(y)))
    two = O.residual_stack_forward([bw, bw], [nw, nw], x, 1e-6)
    assert np.array_equal(two, O.layer_ffn_forward(bw, out, nw, 1e-6)[0])


def test_topk_nan_keys_rank_last_and_stay_distinct():
    """A token with NaN scores (a non-finite activation) still selects k distinct, valid
    experts: NaN keys rank after every other key, by index among themselves (the rule the
    device top-k applies, so both pick the same set)."""
    nan, one, two = 0x7FC0, 0x3F80, 0x4000
    keys = np.array([[nan, one, nan, two, nan, nan],
                     [nan] * 6,
                     [two, nan, one, nan, nan, two]], np.uint16)
    idx = O.topk_rows(keys, 4)
    assert idx.tolist() == [[3, 1, 0, 2], [0, 1, 2, 3], [0, 5, 2, 1]]


def test_gemma4_oracle_vs_numpy_restatement():
    """The C oracle's Gemma4 block (f32 router cascade, top-k by logit, GELU SwitchGLU with
    an f32 hidden) against the float64 restatement: same experts in the same order, weights
    and outputs within f32 rounding."""
    import numpy_ref as R
    cfg = S.GEMMA4_STYLE
    bw = S.host_block(cfg, 7)
    rs, pes = S.host_gemma4_scales(cfg, 7)
    x = S.host_x(3, 6, cfg.hidden)
    y, idx, w = O.gemma4_block_forward(bw, rs, pes, x)
    yr, idxr, wr = R.gemma4_block(bw, rs, pes, x)
    assert np.array_equal(idx, idxr)
    np.testing.assert_allclose(w, wr, rtol=1e-5)
    rel = np.abs(y - yr).mean() / np.abs(yr).mean()
    assert rel < 2e-6, rel


def test_softmax_precision_switch():
    """The routing softmax's internal precision is a switch: f32 (default, what the CUDA
    path computes) or bf16 intermediates, for a reference whose precise=false softmax
    computes in the input type. bf16 mode against a restatement in Python: d = bf16(l - m),
    e = bf16(exp(d)), s = bf16(s + e) in element order, p = bf16(e * bf16(1 / s))."""
    rng = np.random.default_rng(5)
    logits = S.f32_to_bf16_bits((rng.standard_normal((6, 128)) * 3).astype(np.float32))
    p32 = O.softmax_rows(logits)

    def rb(v):
        return float(S.bf16_bits_to_f32(S.f32_to_bf16_bits(np.array([v], np.float32)))[0])

    with O.softmax_precision("bf16"):
        p16 = O.softmax_rows(logits)
    assert np.array_equal(O.softmax_rows(logits), p32), "the switch must restore the default"
    lf = S.bf16_bits_to_f32(logits)
    for r in range(logits.shape[0]):
        m = float(lf[r].max())
        e = [rb(O.exp(rb(float(v) - m))) for v in lf[r]]
        s = 0.0
        for v in e:
            s = rb(np.float32(s) + np.float32(v))
        inv = rb(np.float32(1.0) / np.float32(s))
        want = S.f32_to_bf16_bits(np.array([np.float32(v) * np.float32(inv) for v in e], np.float32))
        assert np.array_equal(p16[r], want), f"row {r}"
    assert not np.array_equal(p16, p32), "the two precisions should differ on these rows"
    # the block route runs under the switch too (weights move by at most a few bf16 ulps)
    bw = S.host_block(S.QWEN3_30B_A3B, 1)
    x = S.host_x(7, 4, S.QWEN3_30B_A3B.hidden)
    i32, w32, _, _ = O.route(bw, x)
    with O.softmax_precision("bf16"):
        i16, w16, _, _ = O.route(bw, x)
    d = np.abs(S.bf16_bits_to_f32(w16) - S.bf16_bits_to_f32(w32))
    assert d.max() < 0.05, d.max()
