"""MLX-semantics quantized ops on torch CUDA tensors, executed by libmoe_b200.so.

Mirrors the reference's Array methods (crates/mlx-core/src/ops.rs):
  quantized_matmul(x, w, scales, biases, transpose, group_size, bits)   ops.rs:592-637
  gather_qmm(x, w, scales, biases, lhs_indices, rhs_indices, transpose,
             group_size, bits, sorted_indices)                           ops.rs:830-891
  fast_rms_norm(x, weight, eps)                                          ops.rs:691-701
Failures raise MlxError("<mlx fn> failed (rc=N): reason"), the Error::Mlx message
of crates/mlx-core/src/array.rs:43-49.

Tensor conventions: activations and scales/biases are torch.bfloat16; packed weights
are 32-bit words (torch.int32 holding the uint32 bit patterns, or torch.uint32);
indices are 32-bit integers (uint32 semantics). All tensors live on one CUDA device
and calls are ordered on torch's current stream.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import MlxError, context_for, library

_WORD_DTYPES = {torch.int32} | ({torch.uint32} if hasattr(torch, "uint32") else set())


def _ptr(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _ctx(t: torch.Tensor):
    if not t.is_cuda:
        raise MlxError("moe_b200", 1, "tensors must be on a CUDA device")
    ctx = context_for(t.device.index)
    ctx.bind_stream(torch.cuda.current_stream(t.device).cuda_stream)
    return ctx


def _need(t, dtypes, name):
    if t is None:
        return
    if t.dtype not in dtypes:
        raise MlxError("moe_b200", 1, f"{name}: dtype {t.dtype} not in {sorted(map(str, dtypes))}")
    if not t.is_contiguous():
        raise MlxError("moe_b200", 1, f"{name}: must be contiguous")


def quantized_matmul(x, w, scales, biases=None, transpose=True, group_size=64, bits=4):
    """out[..., N] = x[..., K] @ dequant(w)^T (transpose=True)."""
    _need(x, {torch.bfloat16}, "x")
    _need(w, _WORD_DTYPES, "w")
    _need(scales, {torch.bfloat16}, "scales")
    _need(biases, {torch.bfloat16}, "biases")
    K = x.shape[-1]
    N = w.shape[-2] if transpose else w.shape[-1] * 32 // bits
    lead = x.shape[:-1]
    M = 1
    for d in lead:
        M *= d
    out = torch.empty(*lead, N, dtype=torch.bfloat16, device=x.device)
    ctx = _ctx(x)
    rc = library().moe_quantized_matmul(ctx.handle, _ptr(x), M, K, _ptr(w), _ptr(scales),
                                        _ptr(biases), N, int(bool(transpose)), group_size, bits,
                                        _ptr(out))
    ctx.check("mlx_quantized_matmul", rc)
    return out


def gather_qmm(x, w, scales, biases=None, lhs_indices=None, rhs_indices=None, transpose=True,
               group_size=64, bits=4, sorted_indices=False):
    """MLX gather_qmm: out[b..., M, N] = x[lhs[b]] @ dequant(w[rhs[b]])^T.

    x is [..., M, K]; w is [E, N, K*bits/32]; lhs/rhs index the flattened batch
    dimensions of x and w and broadcast with each other (and with x's batch shape
    when lhs is omitted). The SwitchGLU form (x [T,1,1,K] with rhs [T,k], or
    x [T,k,1,I] with rhs [T,k]) maps onto the kernel without building indices.
    """
    _need(x, {torch.bfloat16}, "x")
    _need(w, _WORD_DTYPES, "w")
    _need(scales, {torch.bfloat16}, "scales")
    _need(biases, {torch.bfloat16}, "biases")
    if not transpose:
        raise MlxError("mlx_gather_qmm", 2, "transpose=false is not implemented")
    if w.dim() != 3:
        raise MlxError("mlx_gather_qmm", 1, "w must be [E, N, K*bits/32]")
    E, N = w.shape[0], w.shape[1]
    K = x.shape[-1]
    M = x.shape[-2] if x.dim() >= 2 else 1
    xb = tuple(x.shape[:-2])
    dev = x.device
    if rhs_indices is None:
        rhs_indices = torch.zeros((), dtype=torch.int32, device=dev)
    if lhs_indices is None:
        bshape = torch.broadcast_shapes(xb, tuple(rhs_indices.shape))
    else:
        bshape = torch.broadcast_shapes(tuple(lhs_indices.shape), tuple(rhs_indices.shape))
    nb = 1
    for d in bshape:
        nb *= d
    lhs_flat = None
    x_repeat = 1
    fast = (lhs_indices is None and M == 1 and len(bshape) >= 1 and
            (xb == bshape or (len(xb) == len(bshape) and xb[:-1] == bshape[:-1] and xb[-1] == 1)))
    rhs_flat = rhs_indices.expand(bshape).reshape(-1).to(torch.int32).contiguous()
    if fast:
        x_repeat = 1 if xb == bshape else bshape[-1]
        batch = nb
    else:
        if lhs_indices is None:
            nxb = 1
            for d in xb:
                nxb *= d
            lhs_b = torch.arange(nxb, device=dev, dtype=torch.int32).reshape(xb if xb else ())
            lhs_b = lhs_b.expand(bshape).reshape(-1)
        else:
            lhs_b = lhs_indices.expand(bshape).reshape(-1).to(torch.int32)
        # one kernel row per (batch element, m): x row = lhs*M + m, weight = rhs
        m = torch.arange(M, device=dev, dtype=torch.int32)
        lhs_flat = (lhs_b[:, None] * M + m[None, :]).reshape(-1).contiguous()
        rhs_flat = rhs_flat[:, None].expand(nb, M).reshape(-1).contiguous()
        batch = nb * M
    out = torch.empty(*bshape, M, N, dtype=torch.bfloat16, device=dev)
    xc = x.contiguous()
    x_rows = xc.numel() // K
    ctx = _ctx(x)
    rc = library().moe_gather_qmm(ctx.handle, _ptr(xc), x_rows, K, x_repeat, _ptr(lhs_flat), _ptr(w),
                                  _ptr(scales), _ptr(biases), E, N, _ptr(rhs_flat), batch, 1,
                                  group_size, bits, int(bool(sorted_indices)), _ptr(out))
    ctx.check("mlx_gather_qmm", rc)
    return out


def fast_rms_norm(x, weight, eps):
    """bf16(bf16(x * rsqrt(mean(x^2) + eps)) * weight) over the last axis."""
    _need(x, {torch.bfloat16}, "x")
    _need(weight, {torch.bfloat16}, "weight")
    dim = x.shape[-1]
    rows = x.numel() // dim if dim else 0
    out = torch.empty_like(x)
    ctx = _ctx(x)
    rc = library().moe_fast_rms_norm(ctx.handle, _ptr(x), _ptr(weight), float(eps), rows, dim,
                                     _ptr(out))
    ctx.check("mlx_fast_rms_norm", rc)
    return out
