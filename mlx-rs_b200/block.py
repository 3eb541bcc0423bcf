"""MoE block objects mirroring the reference's model-side types.

  SwitchLinear      <- SwitchLinear / ExpertLinear (qwen3_moe_python_port.rs:241-335,
                       lfm2_moe_python_port.rs:426-485): gather_qmm over stacked experts
  SparseMoeBlock    <- SparseMoeBlock::forward (qwen3_moe_python_port.rs:420-488)
  MoeFeedForward    <- MoeFeedForward::forward (lfm2_moe_python_port.rs:541-740)
  RmsNorm           <- RmsNorm::forward (crates/mlx-nn/src/rms_norm.rs:30-34)
  MoeStack          <- a stack of blocks with RMSNorm between them

``forward`` of a block is one call of moe_block_forward (include/moe_b200.h): the
router, scoring, top-k, SwitchGLU, combine and shared expert all run in the CUDA
library on torch's current stream.
"""
from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence

import torch

from . import ops
from ._lib import BlockConfig, BlockWeights as _CWeights, MlxError, QWeight as _CQ, library
from .checkpoint import infer_bits  # the shape rule of qwen3_moe_python_port.rs:221-239
from .ops import _ctx, _ptr
from .synth import (SCORING_SIGMOID_BIAS_SELECT, SCORING_SOFTMAX, SCORING_SOFTMAX_BIAS,
                    BlockWeights, MoeConfig, QWeight)


class SwitchLinear:
    """Stacked expert projection: weight [E, N, K*bits/32], scales/biases [E, N, K/gs]."""

    def __init__(self, q: QWeight, group_size: int = 64, bits: int = 4):
        self.weight, self.scales, self.biases = q.w, q.scales, q.biases
        self.group_size = group_size
        self.bits = infer_bits(tuple(q.w.shape), tuple(q.scales.shape), group_size, bits)

    def forward(self, x, indices):
        return ops.gather_qmm(x, self.weight, self.scales, self.biases, None, indices, True,
                              self.group_size, self.bits, False)


def _cq(q: Optional[QWeight]) -> _CQ:
    if q is None:
        return _CQ(None, None, None)
    return _CQ(q.w.data_ptr(), q.scales.data_ptr(), None if q.biases is None else q.biases.data_ptr())


class _Block:
    """Device weights + config of one block, bound to the C structs."""

    def __init__(self, weights: BlockWeights, config: Optional[MoeConfig] = None):
        self.weights = weights
        self.config = config or weights.config
        c = self.config
        self._cfg = BlockConfig(c.hidden, c.num_experts, c.top_k, c.moe_inter, c.shared_inter,
                                c.scoring, int(c.norm_topk_prob), int(c.has_shared_gate),
                                c.group_size, c.bits)
        w = weights
        eb = w.expert_bias.data_ptr() if w.expert_bias is not None else None
        self._wts = _CWeights(_cq(w.router), eb, _cq(w.gate), _cq(w.up), _cq(w.down),
                              _cq(w.shared_gate), _cq(w.shared_up), _cq(w.shared_down),
                              _cq(w.shared_expert_gate))
        self.device = w.router.w.device

    def reserve(self, max_tokens: int):
        ctx = _ctx(self.weights.router.w)
        ctx.check("moe_ctx_reserve", library().moe_ctx_reserve(ctx.handle, C.byref(self._cfg), max_tokens))

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        H = self.config.hidden
        if x.shape[-1] != H:
            raise MlxError("moe_block_forward", 1, f"hidden {x.shape[-1]} != {H}")
        if x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise MlxError("moe_block_forward", 1, "x must be contiguous bf16")
        T = x.numel() // H
        if out is None:
            out = torch.empty_like(x)
        ctx = _ctx(x)
        rc = library().moe_block_forward(ctx.handle, C.byref(self._cfg), C.byref(self._wts), _ptr(x), T,
                                         _ptr(out))
        ctx.check("moe_block_forward", rc)
        return out

    __call__ = forward

    def forward_layer(self, x: torch.Tensor, norm_weight: torch.Tensor, eps: float = 1e-6,
                      out: Optional[torch.Tensor] = None, normed: Optional[torch.Tensor] = None) -> torch.Tensor:
        """The MoE half of a decoder layer, x + block(RmsNorm(x)), with the residual add
        fused into the combine (moe_layer_ffn_forward): post_attention_layernorm /
        ff.forward / residual.add of MoeBlock::forward (qwen3_moe_python_port.rs:736-739),
        ffn_norm / ffn.forward / residual.add of Lfm2Layer::forward
        (lfm2_moe_python_port.rs:856-868)."""
        H = self.config.hidden
        fn = "moe_layer_ffn_forward"
        if x.shape[-1] != H or x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise MlxError(fn, 1, "x must be contiguous bf16 [..., hidden]")
        if norm_weight.dtype != torch.bfloat16 or norm_weight.numel() != H or not norm_weight.is_contiguous():
            raise MlxError(fn, 1, "norm_weight must be contiguous bf16 [hidden]")
        T = x.numel() // H
        if out is None:
            out = torch.empty_like(x)
        ctx = _ctx(x)
        rc = library().moe_layer_ffn_forward(ctx.handle, C.byref(self._cfg), C.byref(self._wts), _ptr(x), T,
                                             _ptr(norm_weight), float(eps),
                                             _ptr(normed) if normed is not None else None, _ptr(out))
        ctx.check(fn, rc)
        return out

    def profile(self, x: torch.Tensor, out: Optional[torch.Tensor] = None):
        """Run the block once with CUDA events between stages (synchronising).
        Returns (out, {stage: ms}, n_active_experts)."""
        H = self.config.hidden
        T = x.numel() // H
        if out is None:
            out = torch.empty_like(x)
        ms = (C.c_float * 8)()
        na = C.c_int32(0)
        ctx = _ctx(x)
        rc = library().moe_block_profile(ctx.handle, C.byref(self._cfg), C.byref(self._wts), _ptr(x), T,
                                         _ptr(out), ms, C.byref(na))
        ctx.check("moe_block_profile", rc)
        names = ("router", "topk", "group", "gate_up", "down", "shared_gate_up", "shared_down", "combine")
        return out, dict(zip(names, list(ms))), int(na.value)

    def router_logits(self, x: torch.Tensor) -> torch.Tensor:
        """Router logits [T, n] bf16 (n = num_experts, plus the shared_expert_gate column
        when the block has one): the gate Linear of qwen3_moe_python_port.rs:436."""
        H, E = self.config.hidden, self.config.num_experts
        n = E + (1 if self.config.shared_inter > 0 and self.config.has_shared_gate else 0)
        T = x.numel() // H
        logits = torch.empty(T, n, dtype=torch.bfloat16, device=x.device)
        ctx = _ctx(x)
        rc = library().moe_block_router_logits(ctx.handle, C.byref(self._cfg), C.byref(self._wts), _ptr(x), T,
                                               _ptr(logits))
        ctx.check("moe_block_router_logits", rc)
        return logits

    def route(self, x: torch.Tensor):
        """(idx [T,k] int32, weights [T,k] bf16, offsets [E+1] int32, perm [T*k] int32)."""
        H, E, k = self.config.hidden, self.config.num_experts, self.config.top_k
        T = x.numel() // H
        idx = torch.empty(T, k, dtype=torch.int32, device=x.device)
        w = torch.empty(T, k, dtype=torch.bfloat16, device=x.device)
        offsets = torch.empty(E + 1, dtype=torch.int32, device=x.device)
        perm = torch.empty(T * k, dtype=torch.int32, device=x.device)
        ctx = _ctx(x)
        rc = library().moe_block_route(ctx.handle, C.byref(self._cfg), C.byref(self._wts), _ptr(x), T,
                                       _ptr(idx), _ptr(w), _ptr(offsets), _ptr(perm))
        ctx.check("moe_block_route", rc)
        return idx, w, offsets, perm


class SparseMoeBlock(_Block):
    """Qwen-style block: softmax router, top-k, optional renorm, SwitchGLU, optional
    sigmoid-gated shared expert (qwen3_moe_python_port.rs:362-488)."""


class MoeFeedForward(_Block):
    """LFM2-style block (lfm2_moe_python_port.rs:513-741). The reference Rust scores with
    softmax(logits + expert_bias); ``scoring=SCORING_SIGMOID_BIAS_SELECT`` selects
    the sigmoid + bias-for-selection routing instead."""

    def __init__(self, weights: BlockWeights, scoring: Optional[int] = None):
        cfg = weights.config
        if scoring is not None and scoring != cfg.scoring:
            from dataclasses import replace
            cfg = replace(cfg, scoring=scoring)
        if cfg.scoring == SCORING_SOFTMAX and weights.expert_bias is not None:
            from dataclasses import replace
            cfg = replace(cfg, scoring=SCORING_SOFTMAX_BIAS)
        super().__init__(weights, cfg)


class Gemma4MoeBlock(_Block):
    """Gemma4 SparseMoeBlock (crates/mlx-models/src/gemma4.rs:1054-1085): Router::forward
    (:906-936: RMSNorm(x) * hidden^-0.5 * scale in f32, top-k by logit, weights
    softmax[idx] / sum * per_expert_scale[idx]) and the GELU SwitchGlu (:1045-1052). The
    block's output is f32, as in the reference (its router and GELU constants are 0-d f32
    arrays). One call of moe_gemma4_block_forward."""

    def __init__(self, weights: BlockWeights, router_scale: torch.Tensor, per_expert_scale: torch.Tensor):
        super().__init__(weights)
        if router_scale.dtype != torch.bfloat16 or per_expert_scale.dtype != torch.bfloat16:
            raise MlxError("moe_gemma4_block_forward", 1, "scale and per_expert_scale must be bf16")
        self.router_scale = router_scale.contiguous()
        self.per_expert_scale = per_expert_scale.contiguous()

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None, routing: bool = False):
        H, k = self.config.hidden, self.config.top_k
        fn = "moe_gemma4_block_forward"
        if x.shape[-1] != H or x.dtype != torch.bfloat16 or not x.is_contiguous():
            raise MlxError(fn, 1, "x must be contiguous bf16 [..., hidden]")
        T = x.numel() // H
        if out is None:
            out = torch.empty(*x.shape, dtype=torch.float32, device=x.device)
        idx = torch.empty(T, k, dtype=torch.int32, device=x.device) if routing else None
        w = torch.empty(T, k, dtype=torch.float32, device=x.device) if routing else None
        ctx = _ctx(x)
        rc = library().moe_gemma4_block_forward(ctx.handle, C.byref(self._cfg), C.byref(self._wts),
                                                _ptr(self.router_scale), _ptr(self.per_expert_scale), _ptr(x), T,
                                                _ptr(out), _ptr(idx), _ptr(w))
        ctx.check(fn, rc)
        return (out, idx, w) if routing else out

    __call__ = forward


class RmsNorm:
    def __init__(self, weight: torch.Tensor, eps: float = 1e-6):
        self.weight, self.eps = weight, eps

    def forward(self, x):
        return ops.fast_rms_norm(x, self.weight, self.eps)

    __call__ = forward


class MoeStack:
    """h = x; for each layer l: if l > 0: h = RmsNorm_l(h); h = block_l(h).
    With ``residual=True`` the decoder layers' FFN halves instead:
    h = h + block_l(RmsNorm_l(h)) for every l (one moe_layer_ffn_forward per layer)."""

    def __init__(self, blocks: Sequence[_Block], norms: Sequence[RmsNorm], residual: bool = False):
        self.blocks, self.norms, self.residual = list(blocks), list(norms), residual
        if residual and any(n is None for n in self.norms):
            raise ValueError("a residual stack needs a norm for every layer")

    def forward(self, x):
        h = x
        for l, blk in enumerate(self.blocks):
            if self.residual:
                n = self.norms[l]
                h = blk.forward_layer(h, n.weight, n.eps)
                continue
            if l > 0:
                h = self.norms[l](h)
            h = blk(h)
        return h

    __call__ = forward


__all__ = ["SwitchLinear", "SparseMoeBlock", "MoeFeedForward", "Gemma4MoeBlock", "RmsNorm", "MoeStack", "infer_bits",
           "SCORING_SOFTMAX", "SCORING_SOFTMAX_BIAS", "SCORING_SIGMOID_BIAS_SELECT"]
