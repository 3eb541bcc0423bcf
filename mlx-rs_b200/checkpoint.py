"""Checkpoint ingestion for the MoE block: MLX-quantized safetensors -> BlockWeights.

Mirrors how the reference loads the block's tensors (no MLX needed):

  * safetensors files (crates/mlx-core/src/safetensors.rs:7, VarBuilder::from_safetensors,
    crates/mlx-nn/src/var_builder.rs:31-46): an 8-byte little-endian header length, a JSON
    header {name: {dtype, shape, data_offsets}}, then the raw little-endian tensor bytes;
    every shard's names go into one map, names are the dot-joined prefixes
    (VarBuilder::pp / get, :61-97); tensors are memory-mapped here, not copied;
  * Qwen-style blocks (SparseMoeBlock::load, qwen3_moe_python_port.rs:394-418):
    ``<layer>.mlp.gate.{weight,scales,biases}`` is the router, the experts are stored one
    by one as ``<layer>.mlp.experts.<e>.<proj>.{weight,scales,biases}`` and stacked along a
    new leading axis in expert order (SwitchLinear::load, :257-309), the optional shared
    expert is ``<layer>.mlp.shared_expert.<proj>.*`` with ``<layer>.mlp.shared_expert_gate.*``;
  * LFM2-style blocks (MoeFeedForward::load, lfm2_moe_python_port.rs:524-540):
    ``<layer>.feed_forward.gate.*`` is the router, the experts come pre-stacked as
    ``<layer>.feed_forward.switch_mlp.<proj>.*`` (ExpertLinear::load, :435-460), and
    ``<layer>.feed_forward.expert_bias`` is optional (added to the router logits before the
    softmax, :559-567);
  * the block shape and quantization come from config.json (Qwen3MoePythonPortConfig /
    Lfm2MoeConfig fields: hidden_size, num_experts or num_local_experts,
    num_experts_per_tok, moe_intermediate_size, shared_expert_intermediate_size,
    norm_topk_prob, quantization.{group_size, bits}); bits are re-inferred from the packed
    and scale shapes as infer_bits does (:221-239).

The device path computes with bf16 scales, biases and expert_bias, the type MLX 4-bit
checkpoints of these models store them in; the reference keeps tensors in their stored
type (VarBuilder::get casts nothing), so a checkpoint with F16 or F32 scales is rounded to
bf16 here (nearest even) and then differs from the reference by that rounding.
"""
from __future__ import annotations

import glob
import json
import os
import struct
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional

import numpy as np

from .synth import (SCORING_SIGMOID_BIAS_SELECT, SCORING_SOFTMAX, SCORING_SOFTMAX_BIAS, BlockWeights, MoeConfig,
                    QWeight, f32_to_bf16_bits)

_DTYPES = {
    "U8": np.uint8, "I8": np.int8, "U16": np.uint16, "I16": np.int16, "U32": np.uint32, "I32": np.int32,
    "U64": np.uint64, "I64": np.int64, "F16": np.float16, "F32": np.float32, "F64": np.float64,
    "BF16": np.uint16,  # kept as raw bf16 bit patterns
}


class CheckpointError(ValueError):
    pass


@dataclass
class _Entry:
    dtype: str
    shape: tuple
    array: np.ndarray


def read_safetensors(path: str) -> Dict[str, _Entry]:
    """name -> (dtype, shape, memory-mapped array) of one safetensors file."""
    with open(path, "rb") as f:
        head = f.read(8)
        if len(head) != 8:
            raise CheckpointError(f"{path}: not a safetensors file")
        (n,) = struct.unpack("<Q", head)
        header = json.loads(f.read(n))
    base = 8 + n
    data = np.memmap(path, dtype=np.uint8, mode="c")  # copy-on-write: writable views, file untouched
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dt = meta["dtype"]
        if dt not in _DTYPES:
            raise CheckpointError(f"{path}: {name} has unsupported dtype {dt}")
        b, e = meta["data_offsets"]
        shape = tuple(meta["shape"])
        arr = data[base + b: base + e].view(_DTYPES[dt]).reshape(shape)
        out[name] = _Entry(dt, shape, arr)
    return out


def write_safetensors(path: str, tensors: Dict[str, np.ndarray], dtypes: Optional[Dict[str, str]] = None):
    """Write numpy arrays as a safetensors file (uint16 arrays are written as BF16 unless
    dtypes says otherwise). For fixtures and for saving converted weights."""
    rev = {np.dtype(np.uint8): "U8", np.dtype(np.int8): "I8", np.dtype(np.uint16): "BF16",
           np.dtype(np.int16): "I16", np.dtype(np.uint32): "U32", np.dtype(np.int32): "I32",
           np.dtype(np.float16): "F16", np.dtype(np.float32): "F32", np.dtype(np.float64): "F64"}
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        a = np.ascontiguousarray(a)
        dt = (dtypes or {}).get(name, rev[a.dtype])
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _to_bf16(e: _Entry) -> np.ndarray:
    if e.dtype == "BF16":
        return np.asarray(e.array)
    return f32_to_bf16_bits(np.asarray(e.array, dtype=np.float32))


def infer_bits(weight_shape, scales_shape, group_size: int, fallback: int) -> int:
    """Bits per element from the packed and scale shapes (qwen3_moe_python_port.rs:221-239)."""
    packed = weight_shape[-1] if len(weight_shape) else 0
    n_groups = scales_shape[-1] if len(scales_shape) else 0
    if packed <= 0 or n_groups <= 0 or group_size <= 0:
        return fallback
    unpacked = n_groups * group_size
    num = packed * 32
    if num % unpacked:
        return fallback
    b = num // unpacked
    return b if b in (2, 4, 8) else fallback


class _Tensors:
    def __init__(self, maps: Iterable[Dict[str, _Entry]]):
        self.t: Dict[str, _Entry] = {}
        for m in maps:
            self.t.update(m)

    def has(self, name):
        return name in self.t

    def get(self, name) -> _Entry:
        if name not in self.t:
            raise CheckpointError(f"missing tensor {name}")
        return self.t[name]

    def qweight(self, prefix) -> QWeight:
        w = self.get(prefix + ".weight")
        if w.dtype not in ("U32", "I32"):
            raise CheckpointError(f"{prefix}.weight is {w.dtype}: not a packed quantized weight")
        s = self.get(prefix + ".scales")
        b = self.get(prefix + ".biases") if self.has(prefix + ".biases") else None
        return QWeight(np.asarray(w.array).view(np.uint32), _to_bf16(s), None if b is None else _to_bf16(b))

    def stacked(self, prefix, proj, n) -> QWeight:
        """Per-expert tensors <prefix>.<e>.<proj>.* stacked along a new axis 0."""
        qs = [self.qweight(f"{prefix}.{e}.{proj}") for e in range(n)]
        return QWeight(np.stack([q.w for q in qs]), np.stack([q.scales for q in qs]),
                       None if qs[0].biases is None else np.stack([q.biases for q in qs]))


def load_config(path: str) -> dict:
    with open(path) as f:
        return json.load(f)


def block_config(cfg: dict, scoring: Optional[int] = None, has_expert_bias: bool = False) -> MoeConfig:
    """Block shape from config.json with the reference's defaults: 8 experts, 2 per token,
    moe_intermediate_size falling back to intermediate_size, group 64 / 4 bits
    (Qwen3MoePythonPortConfig, qwen3_moe_python_port.rs:170-190; llama.rs:36-60).
    Scoring: softmax over the logits, or over logits + expert_bias when the checkpoint has
    one (MoeFeedForward::forward, lfm2_moe_python_port.rs:559-567)."""
    q = cfg.get("quantization") or cfg.get("quantization_config") or {}
    E = cfg.get("num_experts", cfg.get("num_local_experts")) or 8
    inter = cfg.get("moe_intermediate_size") or cfg.get("intermediate_size") or 0
    Is = cfg.get("shared_expert_intermediate_size") or 0
    if scoring is None:
        scoring = SCORING_SOFTMAX_BIAS if has_expert_bias else SCORING_SOFTMAX
    return MoeConfig(int(cfg["hidden_size"]), int(E), int(cfg.get("num_experts_per_tok") or 2), int(inter),
                     int(Is), int(scoring), bool(cfg.get("norm_topk_prob", False)), bool(Is),
                     int(q.get("group_size", 64)), int(q.get("bits", 4)), name=str(cfg.get("model_type", "checkpoint")))


def load_block(tensors: _Tensors, layer_prefix: str, cfg: dict, scoring: Optional[int] = None) -> BlockWeights:
    """The MoE block of one decoder layer (``layer_prefix`` e.g. "model.layers.3").

    Expert count, hidden and intermediate sizes are taken from the tensors' shapes (the
    config's values only name the defaults), bits are inferred from the packed and scale
    shapes of the expert projections like the reference's loaders do."""
    from dataclasses import replace
    if tensors.has(f"{layer_prefix}.mlp.gate.weight"):  # Qwen layout
        base = f"{layer_prefix}.mlp"
        mc = block_config(cfg, scoring, False)
        router = tensors.qweight(f"{base}.gate")
        E = router.w.shape[0]
        exp = f"{base}.experts"
        if tensors.has(f"{exp}.0.gate_proj.weight"):
            gate, up, down = (tensors.stacked(exp, p, E) for p in ("gate_proj", "up_proj", "down_proj"))
        else:  # already stacked (switch_mlp)
            gate, up, down = (tensors.qweight(f"{base}.switch_mlp.{p}") for p in ("gate_proj", "up_proj", "down_proj"))
        bw = BlockWeights(mc, router, gate, up, down, None, extra={"layout": "qwen"})
        if mc.shared_inter:
            bw.shared_gate = tensors.qweight(f"{base}.shared_expert.gate_proj")
            bw.shared_up = tensors.qweight(f"{base}.shared_expert.up_proj")
            bw.shared_down = tensors.qweight(f"{base}.shared_expert.down_proj")
            has_gate = tensors.has(f"{base}.shared_expert_gate.weight")
            if has_gate:
                bw.shared_expert_gate = tensors.qweight(f"{base}.shared_expert_gate")
            mc = replace(mc, shared_inter=int(bw.shared_gate.w.shape[0]), has_shared_gate=has_gate)
    elif tensors.has(f"{layer_prefix}.feed_forward.switch_mlp.gate_proj.weight"):  # LFM2 layout
        base = f"{layer_prefix}.feed_forward"
        has_eb = tensors.has(f"{base}.expert_bias")
        mc = block_config(cfg, scoring, has_eb)
        router = tensors.qweight(f"{base}.gate")
        gate, up, down = (tensors.qweight(f"{base}.switch_mlp.{p}") for p in ("gate_proj", "up_proj", "down_proj"))
        eb = _to_bf16(tensors.get(f"{base}.expert_bias")) if has_eb else None
        if mc.scoring != SCORING_SOFTMAX and eb is None:
            raise CheckpointError(f"{base}: scoring {mc.scoring} needs expert_bias")
        bw = BlockWeights(mc, router, gate, up, down, eb, extra={"layout": "lfm2"})
    else:
        raise CheckpointError(f"{layer_prefix}: no MoE block (mlp.gate or feed_forward.switch_mlp)")
    bits = infer_bits(bw.gate.w.shape, bw.gate.scales.shape, mc.group_size, mc.bits)
    E, I = bw.gate.w.shape[0], bw.gate.w.shape[1]
    H = bw.gate.w.shape[-1] * 32 // bits
    bw.config = replace(mc, num_experts=int(E), moe_inter=int(I), hidden=int(H), bits=int(bits),
                        top_k=min(mc.top_k, int(E)))
    _check(bw)
    return bw


def _check(bw: BlockWeights):
    c = bw.config
    E, H, I, Is = c.num_experts, c.hidden, c.moe_inter, c.shared_inter
    want = {"router": (E, H), "gate": (E, I, H), "up": (E, I, H), "down": (E, H, I)}
    if Is:
        want.update(shared_gate=(Is, H), shared_up=(Is, H), shared_down=(H, Is))
        if c.has_shared_gate:
            want["shared_expert_gate"] = (1, H)
    for name, shape in want.items():
        q = getattr(bw, name)
        bits = infer_bits(q.w.shape, q.scales.shape, c.group_size, c.bits)
        if bits != c.bits:
            raise CheckpointError(f"{name}: packed shape {q.w.shape} / scales {q.scales.shape} give {bits} bits, "
                                  f"the experts have {c.bits}")
        if tuple(q.w.shape[:-1]) != shape[:-1] or q.w.shape[-1] * 32 // c.bits != shape[-1]:
            raise CheckpointError(f"{name}: packed shape {q.w.shape} does not match {shape} at {c.bits} bits")
        gs_shape = shape[:-1] + (shape[-1] // c.group_size,)
        if tuple(q.scales.shape) != gs_shape or (q.biases is not None and tuple(q.biases.shape) != gs_shape):
            raise CheckpointError(f"{name}: scales/biases shape {q.scales.shape} is not {gs_shape}")
    if bw.expert_bias is not None and tuple(bw.expert_bias.shape) != (E,):
        raise CheckpointError(f"expert_bias shape {bw.expert_bias.shape} is not ({E},)")


def moe_layers(tensors: _Tensors, cfg: dict, prefix: str = "model.layers") -> List[int]:
    """Decoder layers with a MoE block: for Qwen configs every decoder_sparse_step-th layer
    (all when unset; Qwen3MoePythonPortConfig::is_moe_layer, qwen3_moe_python_port.rs:192-197),
    for LFM2 the layers whose feed_forward has switch_mlp weights (Lfm2Layer::load,
    lfm2_moe_python_port.rs:819-826); in both cases only layers whose tensors are present."""
    n = int(cfg.get("num_hidden_layers", 0))
    step = cfg.get("decoder_sparse_step") or 0
    out = []
    for i in range(n):
        p = f"{prefix}.{i}"
        if tensors.has(f"{p}.feed_forward.switch_mlp.gate_proj.weight"):
            out.append(i)
        elif tensors.has(f"{p}.mlp.gate.weight") and (step <= 0 or (i + 1) % step == 0):
            out.append(i)
    return out


def open_checkpoint(directory: str) -> (_Tensors, dict):
    files = sorted(glob.glob(os.path.join(directory, "*.safetensors")))
    if not files:
        raise CheckpointError(f"{directory}: no .safetensors files")
    return _Tensors(read_safetensors(f) for f in files), load_config(os.path.join(directory, "config.json"))


def load_blocks(directory: str, layers: Optional[List[int]] = None, scoring: Optional[int] = None,
                prefix: str = "model.layers") -> List[BlockWeights]:
    """MoE blocks of the given decoder layers (default: every MoE layer of the checkpoint)."""
    tensors, cfg = open_checkpoint(directory)
    if layers is None:
        layers = moe_layers(tensors, cfg, prefix)
    return [load_block(tensors, f"{prefix}.{i}", cfg, scoring) for i in layers]


def load_device_blocks(directory: str, device="cuda", layers: Optional[List[int]] = None,
                       scoring: Optional[int] = None, prefix: str = "model.layers"):
    """The checkpoint's MoE blocks as device blocks ready to call: SparseMoeBlock for the
    Qwen layout, MoeFeedForward for the LFM2 layout (weights copied bit for bit)."""
    from .block import MoeFeedForward, SparseMoeBlock
    from .synth import to_device
    out = []
    for bw in load_blocks(directory, layers, scoring, prefix):
        d = to_device(bw, device)
        if bw.extra.get("layout") == "lfm2":
            out.append(MoeFeedForward(d, scoring=bw.config.scoring))
        else:
            out.append(SparseMoeBlock(d))
    return out


__all__ = ["CheckpointError", "read_safetensors", "write_safetensors", "infer_bits", "block_config",
           "load_block", "load_blocks", "load_device_blocks", "moe_layers", "open_checkpoint", "SCORING_SIGMOID_BIAS_SELECT"]
