// route.cuh — device functions of the router (R1) and scoring / top-k (R2-R4), shared
// by the routing kernels (router.cu) and the fused decode kernel (decode.cu).
//
// Router logits must be bit-identical to the CPU oracle (the expert index sets are
// compared bit for bit), so the router GEMV runs on CUDA cores in the canonical fp32
// order: lane l of a warp owns the 32-element chunks c = l, l+32, ... of K and
// accumulates acc = fma(x[e], w[e], acc) over each chunk in element order, with
// w[e] = fma(scale, q, bias); the 32 lane sums are combined by the xor butterfly
// (offsets 16, 8, 4, 2, 1) and lane 0 holds the result.
//
// Reference: Linear::forward -> quantized_matmul (crates/mlx-nn/src/linear.rs:117-128),
// softmax (qwen3_moe_python_port.rs:437), argpartition + slice + take_along_axis
// (:438-441), norm_topk_prob (:442-445); LFM2 expert_bias + softmax
// (lfm2_moe_python_port.rs:559-586, 680-686).
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace moe {

// (a0, a1) = (fma(x.x, w, a0), fma(x.y, w, a1)) as one packed fp32x2 fma, round to
// nearest even in each half.
MOE_DEV void fma2_acc(float& a0, float& a1, float2 x, float w) {
  unsigned long long acc, xx, ww;
  asm("mov.b64 %0, {%1, %2};" : "=l"(acc) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(xx) : "f"(x.x), "f"(x.y));
  asm("mov.b64 %0, {%1, %1};" : "=l"(ww) : "f"(w));
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(xx), "l"(ww));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a0), "=f"(a1) : "l"(acc));
}

// Logits of rows row0 .. row0+NE-1 for tokens t0 .. t0+NT-1 (one warp).
template <int NE, int NT>
MOE_DEV void router_tile(const RouterArgs& a, int row0, int t0, int lane) {
  if (row0 >= a.n_rows) return;
  const int nchunks = a.K >> 5;
  const int wpr = a.K >> 3;
  const int gpr = a.K / a.group_size;

  float acc[NE][NT];
#pragma unroll
  for (int e = 0; e < NE; ++e)
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[e][t] = 0.0f;

  const uint32_t* wrow[NE];
  const uint16_t* srow[NE];
  const uint16_t* brow[NE];
  bool rvalid[NE];
#pragma unroll
  for (int e = 0; e < NE; ++e) {
    const int r = row0 + e;
    rvalid[e] = r < a.n_rows;
    const bool is_gate = r >= a.E;  // the extra row is shared_expert_gate
    const int rr = is_gate ? 0 : r;
    wrow[e] = (is_gate ? a.gate_w : a.w) + (size_t)rr * wpr;
    srow[e] = (is_gate ? a.gate_s : a.s) + (size_t)rr * gpr;
    const uint16_t* bb = is_gate ? a.gate_b : a.b;
    brow[e] = bb ? bb + (size_t)rr * gpr : nullptr;
  }

  for (int c = lane; c < nchunks; c += 32) {
    const int g = (c * 32) / a.group_size;
    float sc[NE], bi[NE];
#pragma unroll
    for (int e = 0; e < NE; ++e) {
      sc[e] = rvalid[e] ? bf2f(__ldg(srow[e] + g)) : 0.0f;
      bi[e] = (rvalid[e] && brow[e]) ? bf2f(__ldg(brow[e] + g)) : 0.0f;
    }
    // one 8-element word at a time (not unrolled: keeps the token rows of a single word
    // in registers, so that more warps fit on an SM to hide the load latency)
#pragma unroll 1
    for (int word = 0; word < 4; ++word) {
      uint32_t wv[NE];
#pragma unroll
      for (int e = 0; e < NE; ++e) wv[e] = rvalid[e] ? __ldg(wrow[e] + (size_t)c * 4 + word) : 0u;
      uint4 xv[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int tok = t0 + t;
        xv[t] = tok < a.T ? __ldg(reinterpret_cast<const uint4*>(a.x + (size_t)tok * a.K + c * 32 + word * 8))
                          : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int el = 0; el < 8; ++el) {
        float wq[NE];
#pragma unroll
        for (int e = 0; e < NE; ++e) {
          const uint32_t wd = wv[e];
          // q as an exact float: the field in the mantissa of 2^23, minus 2^23
          const float q = __fsub_rn(__uint_as_float(((wd >> (4 * el)) & 0xfu) | 0x4b000000u), 8388608.0f);
          wq[e] = __fmaf_rn(sc[e], q, bi[e]);
        }
        if (NT % 2 == 0) {
          // two tokens per packed fp32x2 fma (two independent IEEE fmas, the same result
          // as two scalar fmas)
#pragma unroll
          for (int t = 0; t < NT; t += 2) {
            const uint32_t xa = (el >> 1) == 0 ? xv[t].x : (el >> 1) == 1 ? xv[t].y : (el >> 1) == 2 ? xv[t].z : xv[t].w;
            const uint32_t xb = (el >> 1) == 0 ? xv[t + 1].x : (el >> 1) == 1 ? xv[t + 1].y
                              : (el >> 1) == 2 ? xv[t + 1].z : xv[t + 1].w;
            const float2 xe = make_float2((el & 1) ? bf_hi(xa) : bf_lo(xa), (el & 1) ? bf_hi(xb) : bf_lo(xb));
#pragma unroll
            for (int e = 0; e < NE; ++e) fma2_acc(acc[e][t], acc[e][t + 1], xe, wq[e]);
          }
        } else {
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const uint32_t xw = (el >> 1) == 0 ? xv[t].x : (el >> 1) == 1 ? xv[t].y : (el >> 1) == 2 ? xv[t].z : xv[t].w;
            const float xe = (el & 1) ? bf_hi(xw) : bf_lo(xw);
#pragma unroll
            for (int e = 0; e < NE; ++e) acc[e][t] = __fmaf_rn(xe, wq[e], acc[e][t]);
          }
        }
      }
    }
  }

#pragma unroll
  for (int e = 0; e < NE; ++e)
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      float v = acc[e][t];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
      acc[e][t] = v;
    }
  if (lane == 0) {
#pragma unroll
    for (int e = 0; e < NE; ++e)
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int tok = t0 + t;
        if (rvalid[e] && tok < a.T) a.logits[(size_t)tok * a.n_rows + row0 + e] = f2bf(acc[e][t]);
      }
  }
}

// router_tile for f32 token rows (a.xf) and unrounded f32 logits (a.logits_f32): the
// Gemma4 router, whose input is RMSNorm(x) * root_size * scale in f32
// (gemma4.rs:906-920). Same canonical order as router_tile.
template <int NE, int NT>
MOE_DEV void router_tile_f32(const RouterArgs& a, int row0, int t0, int lane) {
  if (row0 >= a.n_rows) return;
  const int nchunks = a.K >> 5;
  const int wpr = a.K >> 3;
  const int gpr = a.K / a.group_size;
  float acc[NE][NT];
#pragma unroll
  for (int e = 0; e < NE; ++e)
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[e][t] = 0.0f;
  const uint32_t* wrow[NE];
  const uint16_t* srow[NE];
  const uint16_t* brow[NE];
  bool rvalid[NE];
#pragma unroll
  for (int e = 0; e < NE; ++e) {
    const int r = row0 + e;
    rvalid[e] = r < a.n_rows;
    const int rr = r < a.n_rows ? r : 0;
    wrow[e] = a.w + (size_t)rr * wpr;
    srow[e] = a.s + (size_t)rr * gpr;
    brow[e] = a.b ? a.b + (size_t)rr * gpr : nullptr;
  }
  for (int c = lane; c < nchunks; c += 32) {
    const int g = (c * 32) / a.group_size;
    float sc[NE], bi[NE];
#pragma unroll
    for (int e = 0; e < NE; ++e) {
      sc[e] = rvalid[e] ? bf2f(__ldg(srow[e] + g)) : 0.0f;
      bi[e] = (rvalid[e] && brow[e]) ? bf2f(__ldg(brow[e] + g)) : 0.0f;
    }
#pragma unroll 1
    for (int word = 0; word < 4; ++word) {
      uint32_t wv[NE];
#pragma unroll
      for (int e = 0; e < NE; ++e) wv[e] = rvalid[e] ? __ldg(wrow[e] + (size_t)c * 4 + word) : 0u;
      float4 xl[NT], xh[NT];
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const int tok = t0 + t;
        if (tok < a.T) {
          const float4* p = reinterpret_cast<const float4*>(a.xf + (size_t)tok * a.K + c * 32 + word * 8);
          xl[t] = __ldg(p);
          xh[t] = __ldg(p + 1);
        } else {
          xl[t] = xh[t] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
      }
#pragma unroll
      for (int el = 0; el < 8; ++el) {
        float wq[NE];
#pragma unroll
        for (int e = 0; e < NE; ++e) {
          const float q = __fsub_rn(__uint_as_float(((wv[e] >> (4 * el)) & 0xfu) | 0x4b000000u), 8388608.0f);
          wq[e] = __fmaf_rn(sc[e], q, bi[e]);
        }
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const float4 v = el < 4 ? xl[t] : xh[t];
          const int j = el & 3;
          const float xe = j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
#pragma unroll
          for (int e = 0; e < NE; ++e) acc[e][t] = __fmaf_rn(xe, wq[e], acc[e][t]);
        }
      }
    }
  }
#pragma unroll
  for (int e = 0; e < NE; ++e)
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      float v = acc[e][t];
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
      if (lane == 0 && rvalid[e] && t0 + t < a.T) a.logits_f32[(size_t)(t0 + t) * a.n_rows + row0 + e] = v;
    }
}

// (key desc, index asc), with NaN keys after every other key (NaN among NaN by index
// asc): true if (ka, ia) ranks before (kb, ib). A strict total order, so every round of
// the warp arg-max has one winner and the k selected experts are distinct and valid even
// for a token whose logits are NaN (a non-finite activation). Index 0x7fffffff marks "no
// candidate".
MOE_DEV bool ranks_before(float ka, int ia, float kb, int ib) {
  if (ib == 0x7fffffff) return ia != 0x7fffffff;
  if (ia == 0x7fffffff) return false;
  const bool na = ka != ka, nb = kb != kb;
  if (na != nb) return nb;
  if (na) return ia < ib;
  return ka > kb || (ka == kb && ia < ib);
}

// One warp per token. Lane l holds experts l, l+32, ..., l+32*(PL-1). Logits are read
// through L2 (they may have been written by other CTAs of the same grid).
template <int PL>
MOE_DEV void topk_token(const TopkArgs& a, int t, int lane) {
  const uint16_t* lrow = a.logits + (size_t)t * a.n_rows;
  const bool gemma = a.scoring == 3;  // f32 logits, top-k by logit, f32 weights (no bf16 rounding)

  float val[PL], key[PL];
  float l[PL];
  float m = -__int_as_float(0x7f800000);
#pragma unroll
  for (int i = 0; i < PL; ++i) {
    const int e = lane + 32 * i;
    l[i] = 0.0f;
    if (e < a.E) {
      float v = gemma ? __ldcg(a.logits_f32 + (size_t)t * a.n_rows + e) : bf2f(__ldcg(lrow + e));
      if (a.scoring == 1) v = rbf(__fadd_rn(v, bf2f(a.expert_bias[e])));
      l[i] = v;
      m = fmaxf(m, v);
    }
  }
  if (a.scoring == 2) {
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int e = lane + 32 * i;
      val[i] = 0.0f;
      key[i] = 0.0f;
      if (e < a.E) {
        val[i] = rbf(sigmoid_canon(l[i]));
        key[i] = rbf(__fadd_rn(val[i], bf2f(a.expert_bias[e])));
      }
    }
  } else {
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    float ex[PL];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int e = lane + 32 * i;
      ex[i] = 0.0f;
      if (e < a.E) {
        ex[i] = exp_canon(__fsub_rn(l[i], m));
        s = __fadd_rn(s, ex[i]);
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, off));
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      val[i] = gemma ? __fdiv_rn(ex[i], s) : rbf(__fdiv_rn(ex[i], s));
      key[i] = gemma ? l[i] : val[i];
    }
  }

  // k rounds of warp arg-max over the untaken candidates.
  uint32_t taken = 0;
  int my_sel = 0;
  float my_w = 0.0f;
  for (int j = 0; j < a.k; ++j) {
    float bk = 0.0f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const int e = lane + 32 * i;
      if (e < a.E && !((taken >> i) & 1u) && ranks_before(key[i], e, bk, bi)) {
        bk = key[i];
        bi = e;
      }
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const float ok = __shfl_xor_sync(0xffffffffu, bk, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ranks_before(ok, oi, bk, bi)) {
        bk = ok;
        bi = oi;
      }
    }
    // The owner marks the winner taken and broadcasts its weight value.
    float wv = 0.0f;
    if ((bi & 31) == lane) {
#pragma unroll
      for (int i = 0; i < PL; ++i)
        if (i == (bi >> 5)) {
          taken |= 1u << i;
          wv = val[i];
        }
    }
    wv = __shfl_sync(0xffffffffu, wv, bi & 31);
    if (lane == j) {
      my_sel = bi;
      my_w = wv;
    }
  }
  if (gemma) {
    // w = p / sum_j p_j (f32, j in order) * per_expert_scale (gemma4.rs:927-933)
    float d = 0.0f;
    for (int j = 0; j < a.k; ++j) d = __fadd_rn(d, __shfl_sync(0xffffffffu, my_w, j));
    if (lane < a.k) {
      const float w = __fmul_rn(__fdiv_rn(my_w, d), bf2f(a.per_expert_scale[my_sel]));
      a.weights_f32[(size_t)t * a.k + lane] = w;
      if (a.idx) a.idx[(size_t)t * a.k + lane] = (uint32_t)my_sel;
    }
    return;
  }
  if (a.norm_topk_prob) {
    float d = 0.0f;
    for (int j = 0; j < a.k; ++j) d = __fadd_rn(d, __shfl_sync(0xffffffffu, my_w, j));
    d = rbf(d);
    my_w = rbf(__fdiv_rn(my_w, d));
  }
  if (lane < a.k) {
    const uint16_t wb = f2bf(my_w);
    if (a.idx) a.idx[(size_t)t * a.k + lane] = (uint32_t)my_sel;
    if (a.weights) a.weights[(size_t)t * a.k + lane] = wb;
    if (a.packed) a.packed[(size_t)t * a.k + lane] = (uint32_t)my_sel | ((uint32_t)wb << 16);
  }
  if (a.gate_val && lane == 0) a.gate_val[t] = f2bf(sigmoid_canon(bf2f(__ldcg(lrow + a.E))));
}

}  // namespace moe
