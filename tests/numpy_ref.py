"""An independent numpy restatement of the MoE block, used only to cross-check the C oracle.

It follows the same op sequence and bf16 rounding points (qwen3_moe_python_port.rs:420-488,
lfm2_moe_python_port.rs:541-740) but accumulates every dot product in float64 and uses
numpy's exp, so it agrees with the oracle to within bf16 rounding flips, not bit for bit.
Also holds a restatement of the reference's host top-k selector select_top_k
(qwen3_moe_python_port.rs:491-510), used to check the oracle's tie rule.
"""
from __future__ import annotations

import numpy as np

import mlx_rs_b200.synth as S


def bf(a):
    """Round float64/float32 values to bf16 and return them as float64."""
    return S.bf16_bits_to_f32(S.f32_to_bf16_bits(np.asarray(a, dtype=np.float32))).astype(np.float64)


def f(bits):
    return S.bf16_bits_to_f32(bits).astype(np.float64)


def dequant(q: S.QWeight, gs=64, bits=4):
    w = np.asarray(q.w)
    lead = w.shape[:-1]
    epw = 32 // bits
    shifts = (np.arange(epw, dtype=np.uint32) * bits)
    fields = ((w[..., None] >> shifts) & ((1 << bits) - 1)).reshape(*lead, -1).astype(np.float64)
    s = np.repeat(f(q.scales), gs, axis=-1)
    b = np.repeat(f(q.biases), gs, axis=-1) if q.biases is not None else 0.0
    return s * fields + b


def qmm(x, q, gs=64, bits=4):
    return bf(x @ dequant(q, gs, bits).T)


def select_top_k(row, k):
    """Restatement of select_top_k (qwen3_moe_python_port.rs:491-510): insertion into a
    list kept ordered by (value desc, index asc), truncated to k."""
    top = []
    for idx, prob in enumerate(row):
        pos = None
        for i, (ci, cp) in enumerate(top):
            if prob > cp or (prob == cp and idx < ci):
                pos = i
                break
        if pos is not None:
            top.insert(pos, (idx, prob))
            if len(top) > k:
                top.pop()
        elif len(top) < k:
            top.append((idx, prob))
    return top


def softmax_bf(l):
    m = l.max(axis=-1, keepdims=True)
    e = np.exp(l - m)
    return bf(e / e.sum(axis=-1, keepdims=True))


def sigmoid(v):
    return 1.0 / (1.0 + np.exp(-v))


def route(bw: S.BlockWeights, x_bits):
    c = bw.config
    x = f(x_bits)
    logits = qmm(x, bw.router, c.group_size, c.bits)
    if c.scoring == S.SCORING_SOFTMAX:
        val = softmax_bf(logits)
        key = val
    elif c.scoring == S.SCORING_SOFTMAX_BIAS:
        val = softmax_bf(bf(logits + f(bw.expert_bias)))
        key = val
    else:
        val = bf(sigmoid(logits))
        key = bf(val + f(bw.expert_bias))
    T = x.shape[0]
    idx = np.zeros((T, c.top_k), np.uint32)
    w = np.zeros((T, c.top_k))
    for t in range(T):
        sel = [i for i, _ in select_top_k(list(key[t]), c.top_k)]
        idx[t] = sel
        ws = val[t, sel]
        if c.norm_topk_prob:
            ws = bf(ws / bf(ws.sum()))
        w[t] = ws
    return idx, bf(w), logits


def swiglu(g, u):
    return bf(bf(g * bf(sigmoid(g))) * u)


def block_forward(bw: S.BlockWeights, x_bits):
    c = bw.config
    x = f(x_bits)
    idx, w, _ = route(bw, x_bits)
    T, k = idx.shape
    Wg, Wu, Wd = dequant(bw.gate), dequant(bw.up), dequant(bw.down)
    out = np.zeros((T, c.hidden))
    for t in range(T):
        acc = np.zeros(c.hidden)
        for j in range(k):
            e = idx[t, j]
            g = bf(Wg[e] @ x[t])
            u = bf(Wu[e] @ x[t])
            h = swiglu(g, u)
            y = bf(Wd[e] @ h)
            acc = acc + bf(y * w[t, j])
        out[t] = bf(acc)
    if c.shared_inter:
        sg = qmm(x, bw.shared_gate)
        su = qmm(x, bw.shared_up)
        ys = qmm(swiglu(sg, su), bw.shared_down)
        if c.has_shared_gate:
            gate = bf(sigmoid(qmm(x, bw.shared_expert_gate)))
            ys = bf(ys * gate)
        out = bf(out + ys)
    return out, idx, w


def gemma4_block(bw: S.BlockWeights, router_scale_bits, pes_bits, x_bits):
    """The Gemma4 block (gemma4.rs:906-936, 1045-1085) in float64 except where the
    reference rounds to bf16 (the RMSNorm output, the gate/up gather_qmm outputs)."""
    c = bw.config
    x = f(x_bits)
    ms = np.mean(x * x, axis=-1, keepdims=True)
    hn = bf(x / np.sqrt(ms + 1e-6))
    h = hn * (1.0 / np.sqrt(c.hidden)) * f(router_scale_bits)
    logits = h @ dequant(bw.router, c.group_size, c.bits).T
    m = logits.max(axis=-1, keepdims=True)
    p = np.exp(logits - m)
    p = p / p.sum(axis=-1, keepdims=True)
    idx = np.argsort(-logits, axis=-1, kind="stable")[:, :c.top_k]
    w = np.take_along_axis(p, idx, -1)
    w = w / w.sum(-1, keepdims=True) * f(pes_bits)[idx]
    T, k = idx.shape
    out = np.zeros((T, c.hidden))
    for t in range(T):
        for j in range(k):
            e = idx[t, j]
            g = bf(x[t] @ dequant(S.QWeight(bw.gate.w[e], bw.gate.scales[e], bw.gate.biases[e])).T)
            u = bf(x[t] @ dequant(S.QWeight(bw.up.w[e], bw.up.scales[e], bw.up.biases[e])).T)
            gl = 0.5 * g * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (g + 0.044715 * g ** 3)))
            y = (gl * u) @ dequant(S.QWeight(bw.down.w[e], bw.down.scales[e], bw.down.biases[e])).T
            out[t] += y * w[t, j]
    return out, idx.astype(np.uint32), w
