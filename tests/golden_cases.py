"""Golden fixture cases: definitions, (de)serialisation and the checks that replay them.

Fixtures in tests/golden/*.npz are produced by tests/golden/make_golden.py from the CPU
oracle (after cross-checking it against the independent numpy restatement) and hold
every input and output, so the GPU tests can run without the oracle and the CPU tests
can verify that the oracle still reproduces them bit for bit.
"""
from __future__ import annotations

import numpy as np

import mlx_rs_b200.synth as S

BLOCK_CASES = {
    # name: (config, weight seed, tokens)
    "block_qwen_shared": (S.MoeConfig(256, 12, 4, 128, 192, S.SCORING_SOFTMAX, False, True), 31, 6),
    "block_qwen3_renorm": (S.MoeConfig(512, 12, 8, 64, 0, S.SCORING_SOFTMAX, True, False), 32, 9),
    "block_lfm2_sigmoid": (S.MoeConfig(256, 8, 2, 128, 0, S.SCORING_SIGMOID_BIAS_SELECT, True, False), 33, 7),
    "block_lfm2_softmax_bias": (S.MoeConfig(128, 8, 2, 64, 0, S.SCORING_SOFTMAX_BIAS, False, False), 34, 4),
}

_Q = ("router", "gate", "up", "down", "shared_gate", "shared_up", "shared_down", "shared_expert_gate")
_CFG_FIELDS = ("hidden", "num_experts", "top_k", "moe_inter", "shared_inter", "scoring",
               "norm_topk_prob", "has_shared_gate", "group_size", "bits")


def block_to_dict(bw: S.BlockWeights) -> dict:
    d = {"cfg": np.array([int(getattr(bw.config, f)) for f in _CFG_FIELDS], np.int32)}
    for n in _Q:
        q = getattr(bw, n)
        if q is not None:
            d[f"{n}.w"], d[f"{n}.s"], d[f"{n}.b"] = q.w, q.scales, q.biases
    if bw.expert_bias is not None:
        d["expert_bias"] = bw.expert_bias
    return d


def block_from_dict(z) -> S.BlockWeights:
    vals = [int(v) for v in z["cfg"]]
    kw = dict(zip(_CFG_FIELDS, vals))
    kw["norm_topk_prob"] = bool(kw["norm_topk_prob"])
    kw["has_shared_gate"] = bool(kw["has_shared_gate"])
    cfg = S.MoeConfig(**kw)
    qs = {}
    for n in _Q:
        if f"{n}.w" in z:
            qs[n] = S.QWeight(z[f"{n}.w"], z[f"{n}.s"], z[f"{n}.b"])
    return S.BlockWeights(cfg, qs["router"], qs["gate"], qs["up"], qs["down"],
                          z["expert_bias"] if "expert_bias" in z else None,
                          qs.get("shared_gate"), qs.get("shared_up"), qs.get("shared_down"),
                          qs.get("shared_expert_gate"))


def make_all(oracle):
    """name -> dict of arrays, computed by the oracle."""
    out = {}
    for name, (cfg, seed, T) in BLOCK_CASES.items():
        bw = S.host_block(cfg, seed)
        x = S.host_x(seed, T, cfg.hidden)
        y, idx, w = oracle.block_forward(bw, x)
        off, perm = oracle.group_by_expert(idx, cfg.num_experts)
        _, _, logits, _ = oracle.route(bw, x)
        d = block_to_dict(bw)
        d.update(x=x, out=y, idx=idx, weights=w, offsets=off, perm=perm, logits=logits)
        out[name] = d
    rng = np.random.default_rng(40)
    E, N, K, T, k = 8, 128, 256, 10, 2
    q = S._stack(S._qweight(rng, E * N, K, 64, 4), E, N)
    x = S.f32_to_bf16_bits(rng.standard_normal((T, K), dtype=np.float32))
    rhs = rng.integers(0, E, size=(T, k)).astype(np.uint32)
    lhs = rng.integers(0, T, size=7).astype(np.uint32)
    rhs2 = rng.integers(0, E, size=7).astype(np.uint32)
    out["gather_qmm"] = {
        "x": x, "w": q.w, "s": q.scales, "b": q.biases, "rhs": rhs, "lhs": lhs, "rhs2": rhs2,
        "out": oracle.gather_qmm(x, q.w, q.scales, q.biases, rhs, x_repeat=k),
        "out_lhs": oracle.gather_qmm(x, q.w, q.scales, q.biases, rhs2, lhs=lhs),
    }
    qq = S._qweight(rng, 96, 192, 64, 4)
    xm = S.f32_to_bf16_bits(rng.standard_normal((3, 192), dtype=np.float32))
    out["qmm"] = {"x": xm, "w": qq.w, "s": qq.scales, "b": qq.biases,
                  "out": oracle.qmm(xm, qq.w, qq.scales, qq.biases)}
    xr = S.f32_to_bf16_bits(rng.standard_normal((5, 256), dtype=np.float32) * 7)
    wr = S.f32_to_bf16_bits(rng.uniform(0.5, 1.5, 256).astype(np.float32))
    out["rms_norm"] = {"x": xr, "w": wr, "eps": np.array([1e-6], np.float32),
                       "out": oracle.rms_norm(xr, wr, 1e-6)}
    return out


def check_oracle_against_fixture(name: str, z):
    """The oracle reproduces a committed fixture bit for bit."""
    import oracle as O
    if name.startswith("block_"):
        bw = block_from_dict(z)
        y, idx, w = O.block_forward(bw, z["x"])
        assert np.array_equal(idx, z["idx"]), name
        assert np.array_equal(w, z["weights"]), name
        assert np.array_equal(y, z["out"]), name
        off, perm = O.group_by_expert(idx, bw.config.num_experts)
        assert np.array_equal(off, z["offsets"]) and np.array_equal(perm, z["perm"]), name
    elif name == "gather_qmm":
        k = z["rhs"].shape[1]
        assert np.array_equal(O.gather_qmm(z["x"], z["w"], z["s"], z["b"], z["rhs"], x_repeat=k), z["out"])
        assert np.array_equal(O.gather_qmm(z["x"], z["w"], z["s"], z["b"], z["rhs2"], lhs=z["lhs"]), z["out_lhs"])
    elif name == "qmm":
        assert np.array_equal(O.qmm(z["x"], z["w"], z["s"], z["b"]), z["out"])
    elif name == "rms_norm":
        assert np.array_equal(O.rms_norm(z["x"], z["w"], float(z["eps"][0])), z["out"])
    else:
        raise AssertionError(f"unknown fixture {name}")
