"""Seeded synthetic MoE blocks in the MLX affine 4-bit layout.

Distributions (the benchmark configurations of this path): packed weights with every
4-bit field q ~ U{0..15}; bf16 scales ~ |N(0, 0.02)|; biases = -8 * scale (exact in
bf16); router quantized the same way; optional expert_bias ~ N(0, bias_std) in bf16;
activations x ~ N(0, 1) in bf16.

Host generation (numpy PCG64, ``np.random.default_rng(seed)``) draws, in this order:
router, expert_bias (if any), gate, up, down (each: packed words then scales),
shared gate, shared up, shared down, shared_expert_gate. Activations come from
``np.random.default_rng([seed, T])``. Device generation (``device_block``) uses a
seeded torch CUDA generator with the same distributions, for sizes too large to
build on the host; it is not bit-identical to the host generator.
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Optional

import numpy as np

SCORING_SOFTMAX = 0
SCORING_SOFTMAX_BIAS = 1
SCORING_SIGMOID_BIAS_SELECT = 2


@dataclass(frozen=True)
class MoeConfig:
    hidden: int
    num_experts: int
    top_k: int
    moe_inter: int
    shared_inter: int = 0
    scoring: int = SCORING_SOFTMAX
    norm_topk_prob: bool = False
    has_shared_gate: bool = False
    group_size: int = 64
    bits: int = 4
    name: str = ""


# The block shapes of the benchmark configurations.
QWEN15_MOE_A27B = MoeConfig(2048, 60, 4, 1408, 5632, SCORING_SOFTMAX, False, True,
                            name="qwen1.5-moe-a2.7b")
QWEN3_30B_A3B = MoeConfig(2048, 128, 8, 768, 0, SCORING_SOFTMAX, True, False, name="qwen3-30b-a3b")
LFM2_8B_A1B = MoeConfig(2048, 32, 4, 1792, 0, SCORING_SIGMOID_BIAS_SELECT, True, False,
                        name="lfm2-8b-a1b")
# A Gemma4-style block (gemma4.rs Router + GELU SwitchGlu). The reference names no Gemma4
# MoE configuration, so this shape is synthetic: hidden 2048, 64 experts, top-4,
# moe_intermediate 1024.
GEMMA4_STYLE = MoeConfig(2048, 64, 4, 1024, 0, SCORING_SOFTMAX, True, False, name="gemma4-style")


@dataclass
class QWeight:
    w: object          # [..., N, K*bits/32] 32-bit words
    scales: object     # [..., N, K/gs] bf16
    biases: object = None


@dataclass
class BlockWeights:
    config: MoeConfig
    router: QWeight
    gate: QWeight
    up: QWeight
    down: QWeight
    expert_bias: object = None
    shared_gate: Optional[QWeight] = None
    shared_up: Optional[QWeight] = None
    shared_down: Optional[QWeight] = None
    shared_expert_gate: Optional[QWeight] = None
    extra: dict = field(default_factory=dict)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(nan, ((u >> 16) | 0x40).astype(np.uint16), r)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _qweight(rng, rows: int, K: int, gs: int, bits: int) -> QWeight:
    w = rng.integers(0, 2 ** 32, size=(rows, K * bits // 32), dtype=np.uint32)
    s = f32_to_bf16_bits(np.abs(rng.normal(0.0, 0.02, size=(rows, K // gs))).astype(np.float32))
    b = f32_to_bf16_bits(-8.0 * bf16_bits_to_f32(s))
    return QWeight(w, s, b)


def _stack(q: QWeight, E: int, N: int) -> QWeight:
    return QWeight(q.w.reshape(E, N, -1), q.scales.reshape(E, N, -1), q.biases.reshape(E, N, -1))


def host_block(cfg: MoeConfig, seed: int, bias_std: Optional[float] = None) -> BlockWeights:
    """Numpy weights of one block (bf16 as uint16 bits, words as uint32)."""
    rng = np.random.default_rng(seed)
    H, E, I, Is, gs, bits = (cfg.hidden, cfg.num_experts, cfg.moe_inter, cfg.shared_inter,
                             cfg.group_size, cfg.bits)
    router = _qweight(rng, E, H, gs, bits)
    eb = None
    if cfg.scoring != SCORING_SOFTMAX:
        std = 0.5 if bias_std is None else bias_std
        eb = f32_to_bf16_bits(rng.normal(0.0, std, size=E).astype(np.float32))
    gate = _stack(_qweight(rng, E * I, H, gs, bits), E, I)
    up = _stack(_qweight(rng, E * I, H, gs, bits), E, I)
    down = _stack(_qweight(rng, E * H, I, gs, bits), E, H)
    bw = BlockWeights(cfg, router, gate, up, down, eb)
    if Is > 0:
        bw.shared_gate = _qweight(rng, Is, H, gs, bits)
        bw.shared_up = _qweight(rng, Is, H, gs, bits)
        bw.shared_down = _qweight(rng, H, Is, gs, bits)
        if cfg.has_shared_gate:
            bw.shared_expert_gate = _qweight(rng, 1, H, gs, bits)
    return bw


def host_gemma4_scales(cfg: MoeConfig, seed: int):
    """The Gemma4 router's `scale` [H] and `per_expert_scale` [E] (bf16 bits), each
    ~ U(0.5, 1.5) (seeded)."""
    rng = np.random.default_rng([seed, 4])
    rs = f32_to_bf16_bits(rng.uniform(0.5, 1.5, cfg.hidden).astype(np.float32))
    pes = f32_to_bf16_bits(rng.uniform(0.5, 1.5, cfg.num_experts).astype(np.float32))
    return rs, pes


def host_x(seed: int, T: int, H: int) -> np.ndarray:
    rng = np.random.default_rng([seed, T])
    return f32_to_bf16_bits(rng.standard_normal((T, H), dtype=np.float32))


def with_scoring(bw: BlockWeights, scoring: int, bias_seed: int, bias_std: float) -> BlockWeights:
    """Same weights, other routing: add an expert_bias ~ N(0, bias_std) (seeded)."""
    rng = np.random.default_rng([bias_seed, 7])
    eb = f32_to_bf16_bits(rng.normal(0.0, bias_std, size=bw.config.num_experts).astype(np.float32))
    out = replace(bw, config=replace(bw.config, scoring=scoring), expert_bias=eb)
    return out


# ----------------------------------------------------------------------------------
# torch side
# ----------------------------------------------------------------------------------

def _t(a, device):
    import torch
    if a is None:
        return None
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).to(device).view(torch.bfloat16)
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).to(device)
    raise TypeError(a.dtype)


def _q_to(q: Optional[QWeight], device):
    if q is None:
        return None
    return QWeight(_t(q.w, device), _t(q.scales, device), _t(q.biases, device))


def to_device(bw: BlockWeights, device="cuda") -> BlockWeights:
    """Copy numpy block weights to torch tensors on `device` (bit-identical)."""
    return BlockWeights(bw.config, _q_to(bw.router, device), _q_to(bw.gate, device),
                        _q_to(bw.up, device), _q_to(bw.down, device), _t(bw.expert_bias, device),
                        _q_to(bw.shared_gate, device), _q_to(bw.shared_up, device),
                        _q_to(bw.shared_down, device), _q_to(bw.shared_expert_gate, device))


def x_to_device(x: np.ndarray, device="cuda"):
    return _t(x, device)


def bf16_tensor_to_bits(t) -> np.ndarray:
    import torch
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def _dq(gen, rows, K, gs, bits, device, lead=None):
    import torch
    shape_w = (rows, K * bits // 32) if lead is None else (lead, rows, K * bits // 32)
    shape_s = (rows, K // gs) if lead is None else (lead, rows, K // gs)
    w = torch.randint(-2 ** 31, 2 ** 31, shape_w, dtype=torch.int32, device=device, generator=gen)
    s = (torch.randn(shape_s, device=device, generator=gen, dtype=torch.float32) * 0.02).abs()
    s = s.to(torch.bfloat16)
    b = (s.float() * -8.0).to(torch.bfloat16)
    return QWeight(w, s, b)


def device_block(cfg: MoeConfig, seed: int, device="cuda", bias_std: Optional[float] = None):
    """Same distributions, generated on the device (for the large stacked workloads)."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    H, E, I, Is, gs, bits = (cfg.hidden, cfg.num_experts, cfg.moe_inter, cfg.shared_inter,
                             cfg.group_size, cfg.bits)
    router = _dq(gen, E, H, gs, bits, device)
    eb = None
    if cfg.scoring != SCORING_SOFTMAX:
        std = 0.5 if bias_std is None else bias_std
        eb = (torch.randn(E, device=device, generator=gen) * std).to(torch.bfloat16)
    bw = BlockWeights(cfg, router, _dq(gen, I, H, gs, bits, device, E), _dq(gen, I, H, gs, bits, device, E),
                      _dq(gen, H, I, gs, bits, device, E), eb)
    if Is > 0:
        bw.shared_gate = _dq(gen, Is, H, gs, bits, device)
        bw.shared_up = _dq(gen, Is, H, gs, bits, device)
        bw.shared_down = _dq(gen, H, Is, gs, bits, device)
        if cfg.has_shared_gate:
            bw.shared_expert_gate = _dq(gen, 1, H, gs, bits, device)
    return bw


def device_x(seed: int, T: int, H: int, device="cuda"):
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed * 1000003 + T)
    return torch.randn(T, H, device=device, generator=gen).to(torch.bfloat16)


def weight_bytes(cfg: MoeConfig) -> dict:
    """Algorithmic bytes of the quantized tensors (0.5 B per 4-bit element plus
    2 B scale + 2 B bias per group of 64 = 0.5625 B per element)."""
    per = cfg.bits / 8 + 4 / cfg.group_size
    H, E, I, Is = cfg.hidden, cfg.num_experts, cfg.moe_inter, cfg.shared_inter
    return {
        "per_expert": 3 * H * I * per,
        "router": E * H * per,
        "shared": (3 * H * Is * per + (H * per if cfg.has_shared_gate else 0)) if Is else 0,
    }
