"""Helpers shared by the GPU tests: numpy <-> device tensors and block runs."""
from __future__ import annotations

import numpy as np
import torch

import mlx_rs_b200.synth as S
from mlx_rs_b200.block import MoeFeedForward, SparseMoeBlock


def dev_bits(t) -> np.ndarray:
    """bf16 tensor -> uint16 bits; int32 tensor -> uint32 view."""
    t = t.detach().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).cpu().numpy().view(np.uint16)
    if t.dtype == torch.int32:
        return t.cpu().numpy().view(np.uint32)
    raise TypeError(t.dtype)


def to_dev(a):
    return S.x_to_device(a, "cuda") if a is not None else None


def make_block(bw_host: S.BlockWeights):
    bw = S.to_device(bw_host, "cuda")
    cls = SparseMoeBlock
    if bw_host.config.scoring != S.SCORING_SOFTMAX:
        cls = MoeFeedForward
    return cls(bw) if cls is SparseMoeBlock else cls(bw, scoring=bw_host.config.scoring)


def run_block(blk, x_bits):
    x = to_dev(x_bits)
    out = blk.forward(x)
    idx, w, off, perm = blk.route(x)
    torch.cuda.synchronize()
    return dev_bits(out), dev_bits(idx), dev_bits(w), dev_bits(off).view(np.int32), dev_bits(perm)
