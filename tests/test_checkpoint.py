"""Checkpoint ingestion (mlx_rs_b200.checkpoint): MLX-quantized safetensors in the two
layouts the reference loads (Qwen per-expert tensors stacked at load time; LFM2
pre-stacked switch_mlp with expert_bias) round-trip bit-exactly into block weights, and
the loaded block computes what the original does (oracle on CPU, CUDA path on a GPU).
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest

import mlx_rs_b200.synth as S
from mlx_rs_b200 import checkpoint as C

QWEN_SHARED = S.MoeConfig(256, 8, 2, 128, 192, S.SCORING_SOFTMAX, False, True, name="qwen2_moe")
LFM2 = S.MoeConfig(256, 8, 2, 128, 0, S.SCORING_SOFTMAX_BIAS, True, False, name="lfm2_moe")


def _q(prefix, q, out):
    out[prefix + ".weight"] = q.w
    out[prefix + ".scales"] = q.scales
    if q.biases is not None:
        out[prefix + ".biases"] = q.biases


def _write_qwen(d, blocks, layers, cfg, n_layers, shards=2, extra_cfg=None):
    """Per-expert tensors, as MLX Qwen MoE checkpoints store them, split over `shards` files."""
    t = {}
    for L, bw in zip(layers, blocks):
        p = f"model.layers.{L}.mlp"
        _q(p + ".gate", bw.router, t)
        for e in range(cfg.num_experts):
            for name in ("gate", "up", "down"):
                q = getattr(bw, name)
                _q(f"{p}.experts.{e}.{name}_proj", S.QWeight(q.w[e], q.scales[e], q.biases[e]), t)
        if cfg.shared_inter:
            for name in ("gate", "up", "down"):
                _q(f"{p}.shared_expert.{name}_proj", getattr(bw, "shared_" + name), t)
            if bw.shared_expert_gate is not None:
                _q(f"{p}.shared_expert_gate", bw.shared_expert_gate, t)
        t[f"model.layers.{L}.input_layernorm.weight"] = np.ones(cfg.hidden, np.uint16)  # ignored
    names = sorted(t)
    for s in range(shards):
        C.write_safetensors(os.path.join(d, f"model-{s:05d}-of-{shards:05d}.safetensors"),
                            {n: t[n] for n in names[s::shards]})
    conf = {"model_type": cfg.name, "hidden_size": cfg.hidden, "intermediate_size": 4 * cfg.hidden,
            "moe_intermediate_size": cfg.moe_inter, "num_experts": cfg.num_experts,
            "num_experts_per_tok": cfg.top_k, "norm_topk_prob": cfg.norm_topk_prob,
            "num_hidden_layers": n_layers, "quantization": {"group_size": cfg.group_size, "bits": cfg.bits}}
    if cfg.shared_inter:
        conf["shared_expert_intermediate_size"] = cfg.shared_inter
    conf.update(extra_cfg or {})
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(conf, f)


def _write_lfm2(d, blocks, layers, cfg, n_layers, bias_f32=False):
    t, dt = {}, {}
    for L, bw in zip(layers, blocks):
        p = f"model.layers.{L}.feed_forward"
        _q(p + ".gate", bw.router, t)
        for name in ("gate", "up", "down"):
            _q(f"{p}.switch_mlp.{name}_proj", getattr(bw, name), t)
        if bw.expert_bias is not None:
            t[p + ".expert_bias"] = (S.bf16_bits_to_f32(bw.expert_bias) if bias_f32 else bw.expert_bias)
    # a dense feed-forward layer (no switch_mlp) is not a MoE layer
    t["model.layers.0.feed_forward.w1.weight"] = np.zeros((4, 8), np.uint32)
    C.write_safetensors(os.path.join(d, "model.safetensors"), t, dt)
    conf = {"model_type": cfg.name, "hidden_size": cfg.hidden, "moe_intermediate_size": cfg.moe_inter,
            "num_experts": cfg.num_experts, "num_experts_per_tok": cfg.top_k, "norm_topk_prob": cfg.norm_topk_prob,
            "num_hidden_layers": n_layers, "num_dense_layers": 1,
            "quantization": {"group_size": cfg.group_size, "bits": cfg.bits}}
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(conf, f)


def _same(a: S.BlockWeights, b: S.BlockWeights):
    for name in ("router", "gate", "up", "down", "shared_gate", "shared_up", "shared_down", "shared_expert_gate"):
        qa, qb = getattr(a, name), getattr(b, name)
        assert (qa is None) == (qb is None), name
        if qa is None:
            continue
        for f in ("w", "scales", "biases"):
            x, y = getattr(qa, f), getattr(qb, f)
            assert x.dtype == y.dtype and np.array_equal(x, y), (name, f)
    assert (a.expert_bias is None) == (b.expert_bias is None)
    if a.expert_bias is not None:
        assert np.array_equal(a.expert_bias, b.expert_bias)
    ca, cb = a.config, b.config
    for f in ("hidden", "num_experts", "top_k", "moe_inter", "shared_inter", "scoring", "norm_topk_prob",
              "has_shared_gate", "group_size", "bits"):
        assert getattr(ca, f) == getattr(cb, f), f


def test_safetensors_roundtrip_dtypes(tmp_path):
    rng = np.random.default_rng(0)
    t = {"a": rng.integers(0, 2 ** 32, (3, 5), dtype=np.uint32), "b": rng.integers(0, 2 ** 16, (7,), dtype=np.uint16),
         "c": rng.standard_normal((2, 2, 2)).astype(np.float32), "d": np.zeros((0, 4), np.int32)}
    p = str(tmp_path / "x.safetensors")
    C.write_safetensors(p, t, {"b": "F16"})
    r = C.read_safetensors(p)
    assert r["b"].dtype == "F16" and r["a"].dtype == "U32" and r["c"].dtype == "F32"
    for k, v in t.items():
        assert np.array_equal(np.asarray(r[k].array).view(v.dtype), v), k
    raw = open(p, "rb").read()
    n = int.from_bytes(raw[:8], "little")
    assert n % 8 == 0 and json.loads(raw[8:8 + n])["a"]["data_offsets"] == [0, 60]


def test_infer_bits_matches_reference_rule():
    assert C.infer_bits((768, 256), (768, 32), 64, 8) == 4     # 2048 inputs at 4 bits
    assert C.infer_bits((768, 512), (768, 32), 64, 4) == 8
    assert C.infer_bits((768, 128), (768, 32), 64, 4) == 2
    assert C.infer_bits((768, 192), (768, 32), 64, 4) == 4     # 3 bits: not 2/4/8 -> fallback
    assert C.infer_bits((768, 0), (768, 32), 64, 4) == 4
    assert C.infer_bits((768, 100), (768, 33), 64, 4) == 4     # not divisible -> fallback


def test_qwen_per_expert_checkpoint(tmp_path):
    import oracle as O
    blocks = [S.host_block(QWEN_SHARED, 70 + i) for i in range(2)]
    _write_qwen(str(tmp_path), blocks, [0, 1], QWEN_SHARED, 2)
    loaded = C.load_blocks(str(tmp_path))
    assert len(loaded) == 2
    for want, got in zip(blocks, loaded):
        _same(want, got)
    x = S.host_x(71, 5, QWEN_SHARED.hidden)
    y0, _, _ = O.block_forward(blocks[1], x)
    y1, _, _ = O.block_forward(loaded[1], x)
    assert np.array_equal(y0, y1)


def test_qwen_decoder_sparse_step_and_defaults(tmp_path):
    cfg = S.MoeConfig(256, 8, 2, 128, 0, S.SCORING_SOFTMAX, True, False, name="qwen3_moe")
    b = S.host_block(cfg, 72)
    # MoE on layers 1 and 3 only (decoder_sparse_step 2: layer 2's block is not used);
    # num_experts_per_tok absent -> 2
    _write_qwen(str(tmp_path), [b, b, b], [1, 2, 3], cfg, 4, shards=1, extra_cfg={"decoder_sparse_step": 2})
    conf = json.load(open(tmp_path / "config.json"))
    del conf["num_experts_per_tok"]
    json.dump(conf, open(tmp_path / "config.json", "w"))
    tensors, c = C.open_checkpoint(str(tmp_path))
    assert C.moe_layers(tensors, c) == [1, 3]
    got = C.load_blocks(str(tmp_path))
    assert len(got) == 2 and got[0].config.top_k == 2 and got[0].shared_gate is None
    _same(b, got[1])


def test_lfm2_prestacked_checkpoint_with_expert_bias(tmp_path):
    import oracle as O
    bw = S.host_block(LFM2, 73)
    _write_lfm2(str(tmp_path), [bw], [1], LFM2, 2)
    tensors, c = C.open_checkpoint(str(tmp_path))
    assert C.moe_layers(tensors, c) == [1]
    (got,) = C.load_blocks(str(tmp_path))
    _same(bw, got)
    assert got.config.scoring == S.SCORING_SOFTMAX_BIAS
    x = S.host_x(74, 4, LFM2.hidden)
    assert np.array_equal(O.block_forward(bw, x)[0], O.block_forward(got, x)[0])
    # the other scoring on the same checkpoint, chosen by the caller
    (sig,) = C.load_blocks(str(tmp_path), scoring=S.SCORING_SIGMOID_BIAS_SELECT)
    assert sig.config.scoring == S.SCORING_SIGMOID_BIAS_SELECT


def test_lfm2_f32_expert_bias_rounds_to_bf16(tmp_path):
    bw = S.host_block(LFM2, 75)
    _write_lfm2(str(tmp_path), [bw], [1], LFM2, 2, bias_f32=True)
    (got,) = C.load_blocks(str(tmp_path))
    assert got.expert_bias.dtype == np.uint16 and np.array_equal(got.expert_bias, bw.expert_bias)


def test_checkpoint_errors(tmp_path):
    bw = S.host_block(QWEN_SHARED, 76)
    d = str(tmp_path)
    _write_qwen(d, [bw], [0], QWEN_SHARED, 1, shards=1)
    tensors, cfg = C.open_checkpoint(d)
    with pytest.raises(C.CheckpointError, match="no MoE block"):
        C.load_block(tensors, "model.layers.5", cfg)
    # a missing expert tensor
    del tensors.t["model.layers.0.mlp.experts.3.up_proj.scales"]
    with pytest.raises(C.CheckpointError, match="missing tensor"):
        C.load_block(tensors, "model.layers.0", cfg)
    # a router whose packed width does not match the experts' hidden size
    tensors, cfg = C.open_checkpoint(d)
    e = tensors.t["model.layers.0.mlp.gate.weight"]
    tensors.t["model.layers.0.mlp.gate.weight"] = C._Entry(e.dtype, (8, 16), np.asarray(e.array)[:, :16])
    with pytest.raises(C.CheckpointError, match="router"):
        C.load_block(tensors, "model.layers.0", cfg)
    # an unquantized float weight is not a packed one
    tensors, cfg = C.open_checkpoint(d)
    e = tensors.t["model.layers.0.mlp.gate.weight"]
    tensors.t["model.layers.0.mlp.gate.weight"] = C._Entry("BF16", e.shape, np.asarray(e.array).view(np.uint16))
    with pytest.raises(C.CheckpointError, match="not a packed"):
        C.load_block(tensors, "model.layers.0", cfg)
    with pytest.raises(C.CheckpointError, match="no .safetensors"):
        C.open_checkpoint(str(tmp_path / "nothing"))


@pytest.mark.gpu
def test_checkpoint_block_on_gpu_matches_oracle(tmp_path):
    """A Qwen3-30B-A3B-shaped block written as a per-expert checkpoint, loaded and run
    through the CUDA block: bit-exact with the oracle on the original weights."""
    import oracle as O
    from gpu_util import run_block
    from parity import ULP_TOL, assert_close
    cfg = S.QWEN3_30B_A3B
    bw = S.host_block(cfg, 77)
    _write_qwen(str(tmp_path), [bw], [0], cfg, 1, shards=3)
    (blk,) = C.load_device_blocks(str(tmp_path))
    x = S.host_x(78, 16, cfg.hidden)
    out, idx, w, _, _ = run_block(blk, x)
    y, ridx, rw = O.block_forward(bw, x)
    assert np.array_equal(idx.reshape(ridx.shape), ridx), "expert indices differ"
    assert np.array_equal(w.reshape(rw.shape), rw), "combine weights differ"
    assert_close(out.reshape(y.shape), y, "checkpoint block vs oracle", ULP_TOL)


def test_qwen_prestacked_switch_mlp_and_f16_scales(tmp_path):
    """mlx-lm style Qwen checkpoints hold the experts pre-stacked under mlp.switch_mlp; F16
    scales/biases are rounded to bf16 (the device path's type); a config without a
    quantization block takes the reference's defaults (group 64, 4 bits)."""
    cfg = S.MoeConfig(256, 8, 2, 128, 0, S.SCORING_SOFTMAX, True, False, name="qwen3_moe")
    bw = S.host_block(cfg, 80)
    t = {}
    p = "model.layers.0.mlp"
    _q(p + ".gate", bw.router, t)
    f16 = {}
    for name in ("gate", "up", "down"):
        q = getattr(bw, name)
        t[f"{p}.switch_mlp.{name}_proj.weight"] = q.w
        t[f"{p}.switch_mlp.{name}_proj.scales"] = S.bf16_bits_to_f32(q.scales).astype(np.float16)
        t[f"{p}.switch_mlp.{name}_proj.biases"] = S.bf16_bits_to_f32(q.biases).astype(np.float16)
    C.write_safetensors(str(tmp_path / "model.safetensors"), t, f16)
    conf = {"model_type": "qwen3_moe", "hidden_size": 256, "moe_intermediate_size": 128, "num_experts": 8,
            "num_experts_per_tok": 2, "norm_topk_prob": True, "num_hidden_layers": 1}
    json.dump(conf, open(tmp_path / "config.json", "w"))
    (got,) = C.load_blocks(str(tmp_path))
    assert got.config.group_size == 64 and got.config.bits == 4
    for name in ("gate", "up", "down"):
        q, g = getattr(bw, name), getattr(got, name)
        assert np.array_equal(q.w, g.w)
        want = S.f32_to_bf16_bits(S.bf16_bits_to_f32(q.scales).astype(np.float16).astype(np.float32))
        assert np.array_equal(g.scales, want)


def test_mismatched_scale_shape_is_rejected(tmp_path):
    """Scales with fewer groups than the packed width implies: the loader refuses the block."""
    cfg = S.MoeConfig(256, 8, 2, 128, 0, S.SCORING_SOFTMAX, True, False)
    bw = S.host_block(cfg, 81)
    _write_lfm2(str(tmp_path), [S.with_scoring(bw, S.SCORING_SOFTMAX_BIAS, 1, 0.5)], [1], cfg, 2)
    tensors, c = C.open_checkpoint(str(tmp_path))
    e = tensors.t["model.layers.1.feed_forward.switch_mlp.up_proj.scales"]
    tensors.t["model.layers.1.feed_forward.switch_mlp.up_proj.scales"] = C._Entry(e.dtype, (8, 128, 3),
                                                                                np.asarray(e.array)[..., :3])
    with pytest.raises(C.CheckpointError, match="up"):
        C.load_block(tensors, "model.layers.1", c)
