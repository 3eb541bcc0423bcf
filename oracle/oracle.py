"""ctypes wrapper around oracle/libmoe_oracle.so — the CPU oracle of the MoE block.

TEST INFRASTRUCTURE ONLY: imported by tests/, ``__graft_entry__.smoke()`` and the
cpu_baseline / reference arm of ``bench.py``. The product path never imports it.
Parity status: unpinned (MLX is not available; see moe_oracle.h).

All bf16 arrays are numpy ``uint16`` bit patterns.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libmoe_oracle.so")
_lib = None

SCORING_SOFTMAX = 0
SCORING_SOFTMAX_BIAS = 1
SCORING_SIGMOID_BIAS_SELECT = 2


def build() -> str:
    """Compile the oracle with its Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


class _QW(C.Structure):
    _fields_ = [("w", C.c_void_p), ("s", C.c_void_p), ("b", C.c_void_p)]


class _Cfg(C.Structure):
    _fields_ = [(n, C.c_int32) for n in (
        "hidden", "num_experts", "top_k", "moe_inter", "shared_inter", "scoring",
        "norm_topk_prob", "has_shared_gate", "group_size", "bits")]


class _Wts(C.Structure):
    _fields_ = [("router", _QW), ("expert_bias", C.c_void_p), ("gate", _QW), ("up", _QW),
                ("down", _QW), ("shared_gate", _QW), ("shared_up", _QW), ("shared_down", _QW),
                ("shared_expert_gate", _QW)]


def lib():
    global _lib
    if _lib is None:
        src = os.path.join(_HERE, "moe_oracle.c")
        if not os.path.exists(_LIB_PATH) or (
                os.path.exists(src) and os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
            build()
        L = C.CDLL(_LIB_PATH)
        L.oracle_set_softmax_precision.restype = C.c_int
        L.oracle_set_softmax_precision.argtypes = [C.c_int]
        L.oracle_exp.restype = C.c_float
        L.oracle_exp.argtypes = [C.c_float]
        L.oracle_sigmoid.restype = C.c_float
        L.oracle_sigmoid.argtypes = [C.c_float]
        L.oracle_f32_to_bf16.restype = C.c_uint16
        L.oracle_f32_to_bf16.argtypes = [C.c_float]
        L.oracle_dot_canonical.restype = C.c_float
        L.oracle_dot_canonical.argtypes = [C.c_void_p] * 4 + [C.c_int64, C.c_int, C.c_int]
        L.oracle_qmm.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p,
                                 C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_void_p, C.c_int]
        L.oracle_gather_qmm.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_void_p, C.c_int64, C.c_int64, C.c_void_p,
                                        C.c_int64, C.c_int, C.c_int, C.c_void_p, C.c_int]
        L.oracle_softmax_rows.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p]
        L.oracle_topk_rows.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_int, C.c_void_p]
        L.oracle_route.argtypes = [C.POINTER(_Cfg), C.POINTER(_Wts), C.c_void_p, C.c_int64,
                                   C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        L.oracle_group_by_expert.argtypes = [C.c_int64, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                             C.c_void_p]
        L.oracle_rms_norm.argtypes = [C.c_void_p, C.c_void_p, C.c_float, C.c_int64, C.c_int64,
                                      C.c_void_p, C.c_int]
        L.oracle_block_forward.argtypes = [C.POINTER(_Cfg), C.POINTER(_Wts), C.c_void_p, C.c_int64,
                                           C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]
        L.oracle_swiglu.argtypes = [C.c_void_p, C.c_void_p, C.c_int64, C.c_void_p]
        L.oracle_gemma4_block_forward.argtypes = [C.POINTER(_Cfg), C.POINTER(_Wts), C.c_void_p, C.c_void_p,
                                                  C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p, C.c_void_p,
                                                  C.c_int]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data


def _c(a, dt):
    a = np.ascontiguousarray(a)
    assert a.dtype == dt, (a.dtype, dt)
    return a


def _check(rc, name):
    if rc != 0:
        raise RuntimeError(f"{name} failed (rc={rc})")


def exp(x: float) -> float:
    return lib().oracle_exp(x)


class softmax_precision:
    """Context manager: the routing softmax computes with "f32" (default) or "bf16"
    intermediates (see moe_oracle.c, oracle_set_softmax_precision)."""

    def __init__(self, mode: str):
        if mode not in ("f32", "bf16"):
            raise ValueError(mode)
        self.mode = 0 if mode == "f32" else 1

    def __enter__(self):
        self.prev = lib().oracle_set_softmax_precision(self.mode)
        return self

    def __exit__(self, *exc):
        lib().oracle_set_softmax_precision(self.prev)


def sigmoid(x: float) -> float:
    return lib().oracle_sigmoid(x)


def dot_canonical(x, wrow, srow, brow, gs=64, bits=4) -> float:
    x = _c(x, np.uint16); wrow = _c(wrow, np.uint32); srow = _c(srow, np.uint16)
    brow = None if brow is None else _c(brow, np.uint16)
    return lib().oracle_dot_canonical(_p(x), _p(wrow), _p(srow), _p(brow), x.shape[-1], gs, bits)


def qmm(x, w, s, b, gs=64, bits=4, nthreads=0):
    """bf16(x @ dequant(w).T) — x [M,K] u16, w [N,K*bits/32] u32, s/b [N,K/gs] u16."""
    x = _c(x, np.uint16); w = _c(w, np.uint32); s = _c(s, np.uint16)
    b = None if b is None else _c(b, np.uint16)
    M, K = x.shape
    N = w.shape[0]
    out = np.empty((M, N), np.uint16)
    _check(lib().oracle_qmm(_p(x), M, K, _p(w), _p(s), _p(b), N, gs, bits, _p(out), nthreads),
           "oracle_qmm")
    return out


def gather_qmm(x, w, s, b, rhs, x_repeat=1, lhs=None, gs=64, bits=4, nthreads=0):
    """out[i] = bf16(x[row(i)] @ dequant(w[rhs[i]]).T), row(i) = lhs[i] or i // x_repeat."""
    x = _c(x, np.uint16); w = _c(w, np.uint32); s = _c(s, np.uint16)
    b = None if b is None else _c(b, np.uint16)
    rhs = _c(rhs.reshape(-1), np.uint32)
    lhs = None if lhs is None else _c(lhs.reshape(-1), np.uint32)
    K = x.shape[-1]
    E, N = w.shape[0], w.shape[1]
    batch = rhs.shape[0]
    out = np.empty((batch, N), np.uint16)
    _check(lib().oracle_gather_qmm(_p(x), K, x_repeat, _p(lhs), _p(w), _p(s), _p(b), E, N,
                                   _p(rhs), batch, gs, bits, _p(out), nthreads),
           "oracle_gather_qmm")
    return out


def softmax_rows(logits):
    logits = _c(logits, np.uint16)
    out = np.empty_like(logits)
    _check(lib().oracle_softmax_rows(_p(logits), logits.shape[0], logits.shape[1], _p(out)),
           "oracle_softmax_rows")
    return out


def topk_rows(keys, k):
    keys = _c(keys, np.uint16)
    rows, E = keys.shape
    idx = np.empty((rows, k), np.uint32)
    _check(lib().oracle_topk_rows(_p(keys), rows, E, k, _p(idx)), "oracle_topk_rows")
    return idx


def rms_norm(x, w, eps, nthreads=0):
    x = _c(x, np.uint16); w = _c(w, np.uint16)
    out = np.empty_like(x)
    _check(lib().oracle_rms_norm(_p(x), _p(w), eps, x.shape[0], x.shape[1], _p(out), nthreads),
           "oracle_rms_norm")
    return out


def group_by_expert(idx, E):
    idx = _c(idx, np.uint32)
    T, k = idx.shape
    offsets = np.empty(E + 1, np.int32)
    perm = np.empty(T * k, np.uint32)
    _check(lib().oracle_group_by_expert(T, k, E, _p(idx), _p(offsets), _p(perm)),
           "oracle_group_by_expert")
    return offsets, perm


@dataclass
class _Keep:
    cfg: _Cfg
    wts: _Wts
    arrays: list


def _pack(block):
    """Build the C structs from a block of numpy weights (synth.BlockWeights layout)."""
    c = block.config
    cfg = _Cfg(c.hidden, c.num_experts, c.top_k, c.moe_inter, c.shared_inter, c.scoring,
               int(c.norm_topk_prob), int(c.has_shared_gate), c.group_size, c.bits)
    keep = []

    def qw(q):
        if q is None:
            return _QW(None, None, None)
        arrs = [_c(q.w, np.uint32), _c(q.scales, np.uint16),
                None if q.biases is None else _c(q.biases, np.uint16)]
        keep.extend(a for a in arrs if a is not None)
        return _QW(*[_p(a) for a in arrs])

    eb = None if block.expert_bias is None else _c(block.expert_bias, np.uint16)
    if eb is not None:
        keep.append(eb)
    wts = _Wts(qw(block.router), _p(eb), qw(block.gate), qw(block.up), qw(block.down),
               qw(block.shared_gate), qw(block.shared_up), qw(block.shared_down),
               qw(block.shared_expert_gate))
    return _Keep(cfg, wts, keep)


def route(block, x, nthreads=0):
    """Returns (idx [T,k] u32, weights [T,k] u16, logits [T,E] u16, scores [T,E] u16)."""
    kp = _pack(block)
    x = _c(x, np.uint16)
    T = x.shape[0]
    E, K = block.config.num_experts, block.config.top_k
    idx = np.empty((T, K), np.uint32)
    w = np.empty((T, K), np.uint16)
    logits = np.empty((T, E), np.uint16)
    scores = np.empty((T, E), np.uint16)
    _check(lib().oracle_route(C.byref(kp.cfg), C.byref(kp.wts), _p(x), T, _p(idx), _p(w),
                              _p(logits), _p(scores), nthreads), "oracle_route")
    return idx, w, logits, scores


def block_forward(block, x, nthreads=0):
    """Returns (out [T,H] u16, idx [T,k] u32, weights [T,k] u16)."""
    kp = _pack(block)
    x = _c(x, np.uint16)
    T, H = x.shape
    K = block.config.top_k
    out = np.empty((T, H), np.uint16)
    idx = np.empty((T, K), np.uint32)
    w = np.empty((T, K), np.uint16)
    _check(lib().oracle_block_forward(C.byref(kp.cfg), C.byref(kp.wts), _p(x), T, _p(out),
                                      _p(idx), _p(w), nthreads), "oracle_block_forward")
    return out, idx, w


def gemma4_block_forward(block, router_scale, per_expert_scale, x, nthreads=0):
    """The Gemma4 MoE block (gemma4.rs:1063-1085). Returns (out [T,H] f32, idx [T,k] u32,
    weights [T,k] f32)."""
    kp = _pack(block)
    x = _c(x, np.uint16)
    rs = _c(router_scale, np.uint16)
    pes = _c(per_expert_scale, np.uint16)
    T, H = x.shape
    K = block.config.top_k
    out = np.empty((T, H), np.float32)
    idx = np.empty((T, K), np.uint32)
    w = np.empty((T, K), np.float32)
    _check(lib().oracle_gemma4_block_forward(C.byref(kp.cfg), C.byref(kp.wts), _p(rs), _p(pes), _p(x), T,
                                             _p(out), _p(idx), _p(w), nthreads), "oracle_gemma4_block_forward")
    return out, idx, w


def stack_forward(blocks, norm_weights, x, eps=1e-6, nthreads=0):
    """Stack of blocks with RMSNorm between them: h = x; for l: if l > 0: h = rms_norm(h, w_l);
    h = block_l(h)."""
    h = x
    for l, blk in enumerate(blocks):
        if l > 0:
            h = rms_norm(h, norm_weights[l], eps, nthreads)
        h, _, _ = block_forward(blk, h, nthreads)
    return h


def layer_ffn_forward(block, x, norm_weight, eps=1e-6, nthreads=0):
    """The MoE half of a decoder layer: x + block(rms_norm(x)), the add in fp32 of the two
    bf16 values rounded to bf16 (residual.add(ff.forward(post_attention_layernorm(x))),
    qwen3_moe_python_port.rs:736-739; lfm2_moe_python_port.rs:856-868).
    Returns (out, normed, idx, weights)."""
    h = rms_norm(x, norm_weight, eps, nthreads)
    y, idx, w = block_forward(block, h, nthreads)
    xs = np.asarray(x, np.uint16).reshape(np.shape(y))
    out = (_rbf(_f(xs) + _f(np.asarray(y, np.uint16))).view(np.uint32) >> 16).astype(np.uint16)
    return out, h, idx, w


def residual_stack_forward(blocks, norm_weights, x, eps=1e-6, nthreads=0):
    """Decoder layers' FFN halves in sequence: h = h + block_l(rms_norm(h, w_l))."""
    h = x
    for blk, w in zip(blocks, norm_weights):
        h, _, _, _ = layer_ffn_forward(blk, h, w, eps, nthreads)
    return h


# ----------------------------------------------------------------------------------
# Expert parallelism: the block split over ranks by expert range (the reference runs on
# one device; this restates its combine, qwen3_moe_python_port.rs:471-472, with the
# k-term fp32 sum split by rank and the ranks' partial sums added in rank order).
# ----------------------------------------------------------------------------------

def _f(bits):
    return (bits.astype(np.uint32) << 16).view(np.float32)


def _rbf(v):
    """Round float32 values to bf16 and back (ties to even)."""
    b = v.astype(np.float32).view(np.uint32)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint32)
    nan = np.isnan(v)
    r[nan] = (b[nan] >> 16) | 0x40
    return (r << 16).view(np.float32)


def swiglu(g, u):
    g = _c(g, np.uint16)
    u = _c(u, np.uint16)
    h = np.empty_like(g)
    _check(lib().oracle_swiglu(_p(g), _p(u), g.size, _p(h)), "oracle_swiglu")
    return h


def pack_routing(idx, weights):
    """[T, k] expert | bf16 weight << 16 (the expert-parallel routing record)."""
    return (idx.astype(np.uint32) | (weights.astype(np.uint32) << 16)).astype(np.uint32)


def ep_partials(block_local, x_all, packed_all, expert_begin, num_local, nthreads=0):
    """partial[t] (float32) = sum over j in order, of the pairs whose expert lies in
    [expert_begin, expert_begin + num_local), of bf16(y * w); block_local holds those
    experts' gate/up/down ([num_local, N, K/8])."""
    x_all = _c(x_all, np.uint16)
    T, H = x_all.shape
    k = packed_all.shape[1]
    e = (packed_all & 0xFFFF).astype(np.int64) - expert_begin
    w = (packed_all >> 16).astype(np.uint16)
    local = (e >= 0) & (e < num_local)
    flat = np.flatnonzero(local.reshape(-1))
    partial = np.zeros((T, H), np.float32)
    if flat.size == 0:
        return partial
    t = (flat // k).astype(np.uint32)
    el = e.reshape(-1)[flat].astype(np.uint32)
    b = block_local
    g = gather_qmm(x_all, b.gate.w, b.gate.scales, b.gate.biases, el, lhs=t, nthreads=nthreads)
    u = gather_qmm(x_all, b.up.w, b.up.scales, b.up.biases, el, lhs=t, nthreads=nthreads)
    h = swiglu(g, u)
    y = gather_qmm(h, b.down.w, b.down.scales, b.down.biases, el, x_repeat=1, nthreads=nthreads)
    yf = _f(y)
    wf = _f(w.reshape(-1)[flat])
    j = flat % k
    for jj in range(k):
        sel = np.flatnonzero(j == jj)
        if sel.size:
            partial[t[sel]] = partial[t[sel]] + _rbf(yf[sel] * wf[sel, None])
    return partial


def ep_finish(received, norm_weight=None, eps=1e-6):
    """out = bf16(sum over ranks in order of received[s]); with norm_weight also
    rms_norm(out) (returns (out, normed))."""
    acc = np.zeros(received.shape[1:], np.float32)
    for s in range(received.shape[0]):
        acc = acc + received[s].astype(np.float32)
    b = acc.view(np.uint32)
    out = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    normed = rms_norm(out, norm_weight, eps) if norm_weight is not None else None
    return out, normed
