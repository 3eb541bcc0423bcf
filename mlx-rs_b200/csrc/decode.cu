// decode.cu — the MoE block for decode-sized batches (T <= 8 tokens) in ONE persistent
// cooperative kernel.
//
// Replaces, for small T, the router -> top-k -> grouping -> gate/up -> down -> combine
// launch chain of moe_block_forward (SparseMoeBlock::forward,
// qwen3_moe_python_port.rs:420-488; MoeFeedForward::forward, lfm2_moe_python_port.rs:
// 541-740). At decode sizes that chain is latency-bound: every launch boundary costs
// microseconds while the whole block streams ~21-39 MB (3-6 us at HBM speed). Here one
// CTA per SM runs four phases separated by two grid barriers:
//
//   1. router logits (the canonical-order warp kernel of route.cuh, rows spread over
//      every warp of the grid) -> global scratch;                 grid barrier
//   2. every CTA: top-k of each token (route.cuh, bit-identical to the routing kernels)
//      and the grouping of the T*k pairs by expert (ascending expert, pairs in order),
//      in shared memory; then units of (selected expert, 8 gate + 8 up rows) and of the
//      shared expert's gate/up rows over all warps of the grid: the warp streams its 16
//      weight rows through a private cp.async ring (the whole K in flight), runs
//      mma.sync.m16n8k16 with the expert's tokens as the 8 columns, and writes
//      SwiGLU(gate, up) to scratch. Meanwhile each CTA prefetches its slice of the
//      selected experts' down weights into L2 (cp.async.bulk.prefetch);  grid barrier
//   3. CTA c owns tiles of 16 hidden rows: its warps split the selected experts (and
//      split K of the shared expert's down projection), each writes bf16(y * w) of its
//      pairs into shared memory, and the CTA sums the k terms of each token in index
//      order (the combine of qwen3_moe_python_port.rs:471-472), adds the gated shared
//      expert (:477-484) and the optional residual, and stores the output rows.
//
// Numerics are those of the multi-kernel path: routing bit-identical (same device
// functions), each expert projection accumulated per group of 64 in the same order as
// the GEMV (qgemv.cu), bf16 rounding after every reference op.
//
// The grid barrier is the sense-reversing counter of cooperative groups: one 32-bit word
// whose top bit flips once per barrier, so it needs no reset between calls. Every wait
// is bounded (globaltimer, 200 ms): on expiry the CTA records a status code and returns
// (the outputs are then invalid and moe_ctx_status reports it). The launch is cooperative,
// which guarantees that every CTA of the grid is resident, so the barrier cannot wait on a
// CTA that has not started.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"
#include "route.cuh"

namespace moe {

namespace {

constexpr int kKC = 4;                        // groups of 64 per ring chunk
constexpr int kRowBytes = kKC * 32;           // one weight row's bytes per chunk
constexpr int kSOff = 16 * kRowBytes;         // scales of a stage: [16 rows][4] bf16
constexpr int kBOff = kSOff + 16 * kKC * 2;   // biases of a stage
constexpr int kStage = kBOff + 16 * kKC * 2;  // 2304 bytes
// Ring stages per warp: gate/up (HBM stream) and down (from L2). 8-warp CTAs hold the
// whole K of a unit in flight; 16-warp CTAs (for more units than 8 warps per SM cover)
// half of it.
__host__ __device__ constexpr int ns2_of(int warps) { return warps == 16 ? 4 : 8; }
__host__ __device__ constexpr int ns3_of(int warps) { return warps == 16 ? 2 : 4; }
constexpr uint64_t kWaitNs = 200ull * 1000 * 1000;
constexpr size_t kMaxSmem = 224 * 1024;  // dynamic; the static arrays below take ~1.2 KB

struct DSmem {
  uint32_t xr, x, xsum, tk, ring2, end2, h, hsum, hs, hssum, prod, spart, ring3, end3;
};
__host__ __device__ inline uint32_t al16(uint32_t v) { return (v + 15u) & ~15u; }
// Phases 1-2 and phase 3 reuse the same dynamic shared memory; the top-k scratch (tk)
// lives in the phase-2 rings, which are idle until the top-k is done.
__host__ __device__ inline DSmem dsmem(int T, int P, int E, int H, int I, int Is, int warps) {
  DSmem m{};
  uint32_t o = 0;
  m.xr = o;    o = al16(o + (uint32_t)T * H * 2);              // raw token rows (swizzled pieces)
  m.x = o;     o = al16(o + (uint32_t)T * (2 * H + 16));       // token rows, fragment order
  m.xsum = o;  o = al16(o + (uint32_t)(H / 64) * 8 * 4);       // [G_H][8] group sums
  m.ring2 = o; o = al16(o + (uint32_t)warps * ns2_of(warps) * kStage);
  m.end2 = o;
  m.tk = m.ring2;                                              // [2][T][E] f32 + [16] + [2][P]
  o = 0;
  m.h = o;     o = al16(o + (uint32_t)P * (2 * I + 16));       // SwiGLU rows of the pairs
  m.hsum = o;  o = al16(o + (uint32_t)(I / 64) * P * 4);       // [G_I][P]
  m.hs = o;    o = al16(o + (Is ? (uint32_t)T * (2 * Is + 16) : 0u));
  m.hssum = o; o = al16(o + (Is ? (uint32_t)(Is / 64) * 8 * 4 : 0u));
  m.prod = o;  o = al16(o + (uint32_t)P * 16 * 4);             // bf16(y * w) per pair, 16 rows
  m.spart = o; o = al16(o + (Is ? (uint32_t)warps * 8 * 16 * 4 : 0u));
  m.ring3 = o; o = al16(o + (uint32_t)warps * ns3_of(warps) * kStage);
  m.end3 = o;
  (void)E;
  return m;
}
__host__ __device__ inline uint32_t tk_bytes(int T, int P, int E) {
  return (uint32_t)(2 * T * E * 4 + 16 * 4 + 2 * P * 4);
}
// 16-byte piece p of a raw token row is stored at piece p ^ ((p >> 3) & 7): the router's
// lanes (chunk l = lane, word w: piece 4l + w) then read distinct bank groups.
MOE_DEV uint32_t xr_piece(int p) { return (uint32_t)((p ^ ((p >> 3) & 7)) * 16); }

// mma.sync bf16 m16n8k16 with fp32 accumulate. Not volatile: a pure function of its
// registers, so the compiler may interleave the MMA chains of independent groups.
MOE_DEV void mma_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                     uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
MOE_DEV void mma_first(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                       uint32_t b1) {
  const float z = 0.0f;
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(z));
}
// bf16 pair (128 + q_j, 128 + q_{j+4}) from nibbles j and j+4 of w (exact).
MOE_DEV uint32_t nib_pair(uint32_t w, int j) {
  uint32_t r;
  const uint32_t v = w >> (4 * j);
  asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(r) : "r"(v), "r"(0x000f000fu), "r"(0x43004300u));
  return r;
}
MOE_DEV uint4 lds_u4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
MOE_DEV uint2 lds_u2(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
MOE_DEV void sts_u2(uint32_t a, uint32_t x, uint32_t y) {
  asm volatile("st.shared.v2.u32 [%0], {%1,%2};\n" ::"r"(a), "r"(x), "r"(y) : "memory");
}
MOE_DEV void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
}
MOE_DEV void cp_async8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(dst), "l"(src));
}
MOE_DEV void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(src));
}
MOE_DEV void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
MOE_DEV void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
MOE_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}
MOE_DEV uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Hint: bring [p, p + bytes) into L2 (16-byte aligned, bytes a multiple of 16).
MOE_DEV void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(p), "r"(bytes) : "memory");
}

// Grid-wide barrier (every thread of every CTA calls it). Returns false on every thread
// of a CTA whose wait expired; that CTA records status code 16 and must return.
MOE_DEV bool grid_barrier(uint32_t* bar, int32_t* status, int* ok_s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t nb = blockIdx.x == 0 ? 0x80000000u - (gridDim.x - 1) : 1u;
    __threadfence();
    const uint32_t old = atomicAdd(bar, nb);
    int ok = 1;
    if (((old ^ ld_acquire(bar)) & 0x80000000u) == 0) {
      const uint64_t t0 = global_ns();
      while (((old ^ ld_acquire(bar)) & 0x80000000u) == 0) {
        __nanosleep(64);
        if (global_ns() - t0 > kWaitNs) {
          ok = 0;
          atomicOr(status, 16);
          break;
        }
      }
    }
    __threadfence();
    *ok_s = ok;
  }
  __syncthreads();
  return *ok_s != 0;
}

// Stages nrows rows of K bf16 into shared rows of 2K + 16 bytes in the MMA fragment order
// of the GEMV (qgemv.cu): for each group of 64 and quarter c, elements
// 16c + {0,4,8,12, 1,5,9,13, 2,6,10,14, 3,7,11,15} as bf16 pairs; and the rows' per-group
// sums into sums[g * sstride + r]. Rows come from global memory (row r at src + r * K,
// read through L2: other CTAs of this grid may have written them) or, with FROM_XR, from
// the swizzled raw copy at byte offset xr of the shared array (rows of 2K bytes). Every
// thread calls it.
template <bool FROM_XR, int THREADS>
MOE_DEV void stage_rows(unsigned char* smem, uint32_t dst, float* sums, int sstride, const uint16_t* src,
                        uint32_t xr, int nrows, int K) {
  const int G = K >> 6;
  const int units = nrows * G * 4;
  const int rb = 2 * K + 16;
  for (int u0 = 0; u0 < units; u0 += THREADS) {  // uniform trip count (shuffles below)
    const int u = u0 + (int)threadIdx.x;
    const bool v = u < units;
    const int c = u & 3, g = (u >> 2) % G, t = (u >> 2) / G;
    uint32_t in[8];
    if (v) {
      uint4 v0, v1;
      if (FROM_XR) {
        const int p = g * 8 + c * 2;
        v0 = *reinterpret_cast<const uint4*>(smem + xr + t * 2 * K + xr_piece(p));
        v1 = *reinterpret_cast<const uint4*>(smem + xr + t * 2 * K + xr_piece(p + 1));
      } else {
        const uint4* q = reinterpret_cast<const uint4*>(src + (size_t)t * K + g * 64 + c * 16);
        v0 = __ldcg(q);
        v1 = __ldcg(q + 1);
      }
      in[0] = v0.x; in[1] = v0.y; in[2] = v0.z; in[3] = v0.w;
      in[4] = v1.x; in[5] = v1.y; in[6] = v1.z; in[7] = v1.w;
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) in[i] = 0u;
    }
    float ps = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ps = __fadd_rn(__fadd_rn(ps, bf_lo(in[i])), bf_hi(in[i]));
    ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, 1));
    ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, 2));
    if (v) {
      uint4 o0, o1;
      o0.x = __byte_perm(in[0], in[2], 0x5410);
      o0.y = __byte_perm(in[4], in[6], 0x5410);
      o0.z = __byte_perm(in[0], in[2], 0x7632);
      o0.w = __byte_perm(in[4], in[6], 0x7632);
      o1.x = __byte_perm(in[1], in[3], 0x5410);
      o1.y = __byte_perm(in[5], in[7], 0x5410);
      o1.z = __byte_perm(in[1], in[3], 0x7632);
      o1.w = __byte_perm(in[5], in[7], 0x7632);
      uint4* d = reinterpret_cast<uint4*>(smem + dst + (size_t)t * rb + g * 128 + c * 32);
      d[0] = o0;
      d[1] = o1;
      if (c == 0) sums[g * sstride + t] = ps;
    }
  }
}

// Router logits of row `row` for the T tokens (one warp), in the canonical order of
// router_tile (route.cuh): lane l owns the 32-element chunks c = l, l + 32, ... of K,
// fma in element order per chunk, chunks in order, xor butterfly. Up to four chunks'
// weights per lane are loaded before any is used (one memory round trip for K <= 4096);
// the token rows come from the swizzled raw copy in shared memory; NT >= T tokens. The
// logits go to kDecodeLogitReplicas copies ([replica][T][n_rows]): after the grid barrier
// every CTA reads all of them, and 148 CTAs reading the same two or three L2 lines at once
// queue on those lines' L2 slices for several microseconds (measured); CTA b reads copy
// b mod kDecodeLogitReplicas.
template <int NT>
MOE_DEV void router_row(const RouterArgs& a, int row, const unsigned char* xr, int T, int lane, uint16_t* rep) {
  const bool is_gate = row >= a.E;
  const int rr = is_gate ? 0 : row;
  const int K = a.K, wpr = K >> 3, gpr = K / a.group_size, nchunks = K >> 5;
  const uint32_t* w = (is_gate ? a.gate_w : a.w) + (size_t)rr * wpr;
  const uint16_t* sp = (is_gate ? a.gate_s : a.s) + (size_t)rr * gpr;
  const uint16_t* bsel = is_gate ? a.gate_b : a.b;
  const uint16_t* bp = bsel ? bsel + (size_t)rr * gpr : nullptr;
  float acc[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t] = 0.0f;
  for (int c0 = lane; c0 < nchunks; c0 += 32 * 4) {
    uint4 wv[4];
    float sc[4], bi[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = c0 + 32 * i;
      wv[i] = make_uint4(0, 0, 0, 0);
      sc[i] = bi[i] = 0.0f;
      if (c < nchunks) {
        wv[i] = __ldg(reinterpret_cast<const uint4*>(w + (size_t)c * 4));
        const int g = (c * 32) / a.group_size;
        sc[i] = bf2f(__ldg(sp + g));
        bi[i] = bp ? bf2f(__ldg(bp + g)) : 0.0f;
      }
    }
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
      const int c = c0 + 32 * i;
      if (c >= nchunks) break;
      const uint32_t wds[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
#pragma unroll
      for (int word = 0; word < 4; ++word) {
        const uint32_t off = xr_piece(c * 4 + word);
        uint4 xp[NT];
#pragma unroll
        for (int t = 0; t < NT; ++t)
          xp[t] = t < T ? *reinterpret_cast<const uint4*>(xr + t * 2 * K + off) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int el = 0; el < 8; ++el) {
          const float q = __fsub_rn(__uint_as_float(((wds[word] >> (4 * el)) & 0xfu) | 0x4b000000u), 8388608.0f);
          const float wq = __fmaf_rn(sc[i], q, bi[i]);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const uint32_t xw = (el >> 1) == 0 ? xp[t].x : (el >> 1) == 1 ? xp[t].y : (el >> 1) == 2 ? xp[t].z : xp[t].w;
            const float xe = (el & 1) ? bf_hi(xw) : bf_lo(xw);
            acc[t] = __fmaf_rn(xe, wq, acc[t]);
          }
        }
      }
    }
  }
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float v = acc[t];
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
    // every lane holds the sum after the xor butterfly: lanes 0..15 write one replica each
    if (lane < kDecodeLogitReplicas && t < T) rep[((size_t)lane * T + t) * a.n_rows + row] = f2bf(v);
  }
}

// Scoring, top-k and combine weights of the T tokens with every thread of the CTA; the
// results equal topk_token's bit for bit: the same max, exp, canonical-order sum (lane l
// sums experts l, l+32, ... in order, then the xor butterfly), IEEE divides and
// roundings; the expert of rank j (the number of experts ranking before it) is the j-th
// arg-max round's winner. sel/selw: [T*k] scratch; red: [16] floats.
template <int THREADS>
MOE_DEV void topk_cta(const TopkArgs& a, int T, float* vals, float* keys, float* red, int* sel, float* selw,
                      uint32_t* s_idx, uint16_t* s_w, uint16_t* s_gate, bool has_gate) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int E = a.E, n = T * E, k = a.k;
  for (int i = tid; i < n; i += THREADS) {
    const int t = i / E, e = i - t * E;
    float v = bf2f(__ldcg(a.logits + (size_t)t * a.n_rows + e));
    if (a.scoring == 1) v = rbf(__fadd_rn(v, bf2f(a.expert_bias[e])));
    if (a.scoring == 2) {
      const float sv = rbf(sigmoid_canon(v));
      vals[i] = sv;
      keys[i] = rbf(__fadd_rn(sv, bf2f(a.expert_bias[e])));
    } else {
      vals[i] = v;
    }
  }
  if (has_gate && tid < T) s_gate[tid] = f2bf(sigmoid_canon(bf2f(__ldcg(a.logits + (size_t)tid * a.n_rows + E))));
  __syncthreads();
  if (a.scoring != 2) {
    if (warp < T) {
      float m = -__int_as_float(0x7f800000);
      for (int e = lane; e < E; e += 32) m = fmaxf(m, vals[warp * E + e]);
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
      if (lane == 0) red[warp] = m;
    }
    __syncthreads();
    for (int i = tid; i < n; i += THREADS) vals[i] = exp_canon(__fsub_rn(vals[i], red[i / E]));
    __syncthreads();
    if (warp < T) {
      float sm = 0.0f;
      for (int e = lane; e < E; e += 32) sm = __fadd_rn(sm, vals[warp * E + e]);
#pragma unroll
      for (int off = 16; off >= 1; off >>= 1) sm = __fadd_rn(sm, __shfl_xor_sync(0xffffffffu, sm, off));
      if (lane == 0) red[8 + warp] = sm;
    }
    __syncthreads();
    for (int i = tid; i < n; i += THREADS) {
      const float v = rbf(__fdiv_rn(vals[i], red[8 + i / E]));
      vals[i] = v;
      keys[i] = v;
    }
  }
  __syncthreads();
  // selection. Every key is a bf16 value, so (key, expert) packs into one 32-bit word
  // whose unsigned order is the order of ranks_before: the key's bits mapped to an
  // order-preserving code in the high half (NaN lowest), 0xffff - expert in the low half
  // (index ascending among equal keys). The expert of rank r (the number of larger words
  // in its token's row) is the r-th winner of topk_token's arg-max rounds.
  uint32_t* ord = reinterpret_cast<uint32_t*>(keys);  // in place: [T][E]
  for (int i = tid; i < n; i += THREADS) {
    const int e = i - (i / E) * E;
    const float kf = keys[i];
    uint32_t b = __float_as_uint(kf) >> 16;  // exact: keys are bf16 values
    if (b == 0x8000u) b = 0u;                 // -0 ties with +0, as in ranks_before
    const uint32_t code = kf != kf ? 0u : ((b & 0x8000u) ? (~b & 0xffffu) : (b | 0x8000u));
    ord[i] = (code << 16) | (0xffffu - (uint32_t)e);
  }
  __syncthreads();
  for (int i = tid; i < n; i += THREADS) {
    const int t = i / E;
    const uint32_t* orow = ord + t * E;
    const uint32_t me = ord[i];
    int r0 = 0, r1 = 0, r2 = 0, r3 = 0;
    int e2 = 0;
    if ((E & 3) == 0) {
      const uint4* o4 = reinterpret_cast<const uint4*>(orow);
      for (; e2 < E; e2 += 4) {
        const uint4 v = o4[e2 >> 2];
        r0 += v.x > me;
        r1 += v.y > me;
        r2 += v.z > me;
        r3 += v.w > me;
      }
    }
    for (; e2 < E; ++e2) r0 += orow[e2] > me;
    const int r = r0 + r1 + r2 + r3;
    if (r < k) {
      sel[t * k + r] = (int)(0xffffu - (me & 0xffffu));
      selw[t * k + r] = vals[i];
    }
  }
  __syncthreads();
  if (tid < T * k) {
    const int t = tid / k;
    float w = selw[tid];
    if (a.norm_topk_prob) {
      float d = 0.0f;
      for (int j = 0; j < k; ++j) d = __fadd_rn(d, selw[t * k + j]);
      d = rbf(d);
      w = rbf(__fdiv_rn(w, d));
    }
    s_idx[tid] = (uint32_t)sel[tid];
    s_w[tid] = f2bf(w);
  }
  __syncthreads();
}

// The 16 weight rows of one unit: ring rows 0-7 are rows row0[0]..+7 of matrix 0, ring
// rows 8-15 rows row0[1]..+7 of matrix 1 (gated: gate and up rows of the same outputs;
// plain: one matrix, row0[1] = row0[0] + 8). Pointers are at the expert's base.
struct Rows {
  const uint32_t* w[2];
  const uint16_t* s[2];
  const uint16_t* b[2];
  int row0[2];
  int N;
};
// The unit's 8 columns: xb = byte offset (in the dynamic shared array) of this lane's B
// row (column gq) in the staging; xs + r0c / r1c:
// the group sums (stride xs_stride) of the staged rows of columns 2cq and 2cq+1.
struct Cols {
  uint32_t xb;
  const float* xs;
  int xs_stride, r0c, r1c;
};

// One warp's sequence of units (unit i = first + i * step, i < count), each 16 weight rows
// over chunks [cb, ce) of 4 groups of a K of G groups (wpr words per row), streamed
// through one NS-stage cp.async ring: the chunks of the next units are in flight while
// the current unit computes. Per unit, acc = the C fragment (MMA rows gq / gq+8, columns
// 2cq / 2cq+1); per group the GEMV's fold s * sum_k x(128 + q) + (b - 128 s) * sum_k x in
// fp32; epi(unit, acc) after the unit's last chunk.
template <int NS, class RowsFn, class ColsFn, class EpiFn>
MOE_DEV void stream_units(const unsigned char* smem, uint32_t sbase, int first, int step, int count, int cb, int ce,
                          int G, int wpr, uint32_t ring, bool scale8, RowsFn rows_of, ColsFn cols_of, EpiFn epi) {
  const int lane = threadIdx.x & 31, gq = lane >> 2, cq = lane & 3;
  const int per = ce - cb;
  const int Q = count * per;
  if (Q <= 0) return;
  const int nch = (G + kKC - 1) / kKC;
  const int tail = G - (nch - 1) * kKC;
  // issue cursor: the unit whose chunks are being copied
  const uint32_t* src[4];
  uint32_t dst[4];
  int pgl[4];
  const uint16_t* ssrc = nullptr;
  const int srr = lane & 15, which = lane >> 4;
  const uint32_t sdst = (which ? kBOff : kSOff) + srr * (kKC * 2);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int q = i * 32 + lane;
    const int rr = q >> 3, part = q & 7, gl = part >> 1, half = part & 1;
    dst[i] = rr * kRowBytes + ((gl ^ (rr & 3)) * 32) + half * 16;
    pgl[i] = gl;
    src[i] = nullptr;
  }
  int iu = -1;
  auto issue = [&](int q) {
    const int i = q / per, c = cb + (q - i * per);
    if (i != iu) {
      iu = i;
      const Rows R = rows_of(first + i * step);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int qq = j * 32 + lane;
        const int rr = qq >> 3, part = qq & 7, m = rr >> 3;
        int row = R.row0[m] + (rr & 7);
        row = row < R.N ? row : R.N - 1;
        src[j] = R.w[m] + (size_t)row * wpr + part * 4 + (size_t)cb * kKC * 8;
      }
      const int sm = srr >> 3;
      int srow = R.row0[sm] + (srr & 7);
      srow = srow < R.N ? srow : R.N - 1;
      const uint16_t* sb = which ? R.b[sm] : R.s[sm];
      ssrc = sb ? sb + (size_t)srow * G + (size_t)cb * kKC : nullptr;
    }
    const uint32_t st = sbase + ring + (uint32_t)((q % NS) * kStage);
    const bool full = c + 1 < nch || tail == kKC;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (full || pgl[j] < tail) cp_async16(st + dst[j], src[j]);
#pragma unroll
    for (int j = 0; j < 4; ++j) src[j] += kKC * 8;
    if (ssrc) {
      if (scale8) {
        cp_async8(st + sdst, ssrc);
      } else {
        cp_async4(st + sdst, ssrc);  // groups 0-1 of the chunk (G is even)
        if (full) cp_async4(st + sdst + 4, ssrc + 2);
      }
      ssrc += kKC;
    } else {
      sts_u2(st + sdst, 0u, 0u);  // no biases
    }
    cp_commit();
  };
#pragma unroll 1
  for (int q = 0; q < NS - 1; ++q) {
    if (q < Q) issue(q);
    else cp_commit();
  }
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  Cols C{};
#pragma unroll 1
  for (int q = 0; q < Q; ++q) {
    if (q + NS - 1 < Q) issue(q + NS - 1);
    else cp_commit();
    const int i = q / per, c = cb + (q - i * per);
    if (c == cb) {
      C = cols_of(first + i * step);
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = 0.0f;
    }
    cp_wait<NS - 1>();
    __syncwarp();
    const unsigned char* st = smem + ring + (q % NS) * kStage;
    const uint2 sw0 = *reinterpret_cast<const uint2*>(st + kSOff + gq * (kKC * 2));
    const uint2 sw1 = *reinterpret_cast<const uint2*>(st + kSOff + (gq + 8) * (kKC * 2));
    const uint2 bw0 = *reinterpret_cast<const uint2*>(st + kBOff + gq * (kKC * 2));
    const uint2 bw1 = *reinterpret_cast<const uint2*>(st + kBOff + (gq + 8) * (kKC * 2));
#pragma unroll
    for (int gl = 0; gl < kKC; ++gl) {
      const int g = c * kKC + gl;
      if (g < G) {
        const uint4 v0 = *reinterpret_cast<const uint4*>(smem + C.xb + g * 128);
        const uint4 v1 = *reinterpret_cast<const uint4*>(smem + C.xb + g * 128 + 16);
        const uint32_t bfr[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        const float X0 = C.xs[g * C.xs_stride + C.r0c], X1 = C.xs[g * C.xs_stride + C.r1c];
        const uint32_t off = ((gl ^ (gq & 3)) * 32) + cq * 8;
        const uint2 wlo = *reinterpret_cast<const uint2*>(st + gq * kRowBytes + off);
        const uint2 whi = *reinterpret_cast<const uint2*>(st + (gq + 8) * kRowBytes + off);
        float d[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t a0 = nib_pair(wlo.x, j), a1 = nib_pair(whi.x, j);
          const uint32_t a2 = nib_pair(wlo.y, j), a3 = nib_pair(whi.y, j);
          if (j == 0) mma_first(d, a0, a1, a2, a3, bfr[0], bfr[1]);
          else mma_acc(d, a0, a1, a2, a3, bfr[2 * j], bfr[2 * j + 1]);
        }
        const uint32_t s02 = (gl >> 1) ? sw0.y : sw0.x, s12 = (gl >> 1) ? sw1.y : sw1.x;
        const uint32_t b02 = (gl >> 1) ? bw0.y : bw0.x, b12 = (gl >> 1) ? bw1.y : bw1.x;
        const float s_l = (gl & 1) ? bf_hi(s02) : bf_lo(s02);
        const float s_h = (gl & 1) ? bf_hi(s12) : bf_lo(s12);
        const float c_l = __fmaf_rn(-128.0f, s_l, (gl & 1) ? bf_hi(b02) : bf_lo(b02));
        const float c_h = __fmaf_rn(-128.0f, s_h, (gl & 1) ? bf_hi(b12) : bf_lo(b12));
        acc[0] = __fmaf_rn(c_l, X0, __fmaf_rn(s_l, d[0], acc[0]));
        acc[1] = __fmaf_rn(c_l, X1, __fmaf_rn(s_l, d[1], acc[1]));
        acc[2] = __fmaf_rn(c_h, X0, __fmaf_rn(s_h, d[2], acc[2]));
        acc[3] = __fmaf_rn(c_h, X1, __fmaf_rn(s_h, d[3], acc[3]));
      }
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
    if (c == ce - 1) epi(first + i * step, acc);
  }
  cp_wait<0>();
  __syncwarp();
}

template <int NT, int WARPS>
__global__ void __launch_bounds__(WARPS * 32, 1) decode_block_kernel(DecodeArgs a) {
  constexpr int kThreads = WARPS * 32, kNS2 = ns2_of(WARPS), kNS3 = ns3_of(WARPS);
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint32_t s_idx[kDecodeMaxP];
  __shared__ uint16_t s_w[kDecodeMaxP];
  __shared__ uint16_t s_gate[kDecodeMaxT];
  __shared__ int s_perm[kDecodeMaxP];
  __shared__ int s_ue[kDecodeMaxP];
  __shared__ int s_ub[kDecodeMaxP + 1];
  __shared__ int s_U;
  __shared__ int s_ok;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, cq = lane & 3;
  const int gw = blockIdx.x * WARPS + warp, W = gridDim.x * WARPS;
  const int T = a.T, k = a.k, P = T * k, H = a.H, I = a.I, Is = a.Is, E = a.ta.E;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
  const DSmem L = dsmem(T, P, E, H, I, Is, WARPS);

  // ---- phase 1: the token rows into shared memory, then router logits, one row per warp
  for (int i = tid; i < T * (H / 8); i += kThreads) {
    const int t = i / (H / 8), p = i - t * (H / 8);
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(a.ra.x) + (size_t)t * (H / 8) + p);
    *reinterpret_cast<uint4*>(smem + L.xr + t * 2 * H + xr_piece(p)) = v;
  }
  __syncthreads();
  for (int row = gw; row < a.ra.n_rows; row += W) router_row<NT>(a.ra, row, smem + L.xr, T, lane, a.logits_rep);
  if (!grid_barrier(a.barrier, a.status, &s_ok)) return;

  // ---- every CTA: scoring / top-k of the tokens, then the grouping of the pairs
  {
    float* vals = reinterpret_cast<float*>(smem + L.tk);
    float* keys = vals + T * E;
    float* red = keys + T * E;
    int* sel = reinterpret_cast<int*>(red + 16);
    float* selw = reinterpret_cast<float*>(sel + P);
    TopkArgs ta = a.ta;
    ta.logits = a.logits_rep + (size_t)(blockIdx.x % kDecodeLogitReplicas) * T * ta.n_rows;
    topk_cta<kThreads>(ta, T, vals, keys, red, sel, selw, s_idx, s_w, s_gate, a.has_gate != 0);
  }
  if (warp == 0) {
    // position of pair p in (expert, p) order
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int p = lane + 32 * h;
      if (p < P) {
        const uint32_t e = s_idx[p];
        int r = 0;
        for (int q = 0; q < P; ++q) {
          const uint32_t eq = s_idx[q];
          r += (eq < e || (eq == e && q < p)) ? 1 : 0;
        }
        s_perm[r] = p;
      }
    }
    __syncwarp();
    bool start[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int pos = lane + 32 * h;
      start[h] = pos < P && (pos == 0 || s_idx[s_perm[pos]] != s_idx[s_perm[pos - 1]]);
    }
    const unsigned m0 = __ballot_sync(0xffffffffu, start[0]), m1 = __ballot_sync(0xffffffffu, start[1]);
    const unsigned lt = (1u << lane) - 1u;
    if (start[0]) {
      const int u = __popc(m0 & lt);
      s_ue[u] = (int)s_idx[s_perm[lane]];
      s_ub[u] = lane;
    }
    if (start[1]) {
      const int u = __popc(m0) + __popc(m1 & lt);
      s_ue[u] = (int)s_idx[s_perm[lane + 32]];
      s_ub[u] = lane + 32;
    }
    if (lane == 0) {
      const int U = __popc(m0) + __popc(m1);
      s_U = U;
      s_ub[U] = P;
      if (blockIdx.x == 0 && a.n_active) *a.n_active = U;
    }
  }
  __syncthreads();
  const int U = s_U;

  // ---- phase 2: gate/up + SwiGLU of the selected experts and the shared expert
  stage_rows<true, kThreads>(smem, L.x, reinterpret_cast<float*>(smem + L.xsum), 8, nullptr, L.xr, T, H);
  {
    // this CTA's slice of every selected expert's down weights (and of the shared down)
    // into L2: the down projection after the next barrier reads L2, not HBM. One thread
    // per (matrix, array) region; 32-bit sizes (a region is at most H * I / 2 bytes).
    const int nreg = 3 * (U + (Is ? 1 : 0));
    if (tid < nreg) {
      const int u = tid / 3, r = tid - u * 3;
      const bool sh = u == U;
      const int e = sh ? 0 : s_ue[u];
      const int wpr = sh ? Is / 8 : I / 8, G = sh ? Is / 64 : I / 64;
      const uint16_t* sa = r == 1 ? (sh ? a.ssd : a.sd) : (sh ? a.sbd : a.bd);
      const char* base = r == 0 ? reinterpret_cast<const char*>((sh ? a.swd : a.wd) + (size_t)e * H * wpr)
                                : (sa ? reinterpret_cast<const char*>(sa + (size_t)e * H * G) : nullptr);
      const uint32_t bytes = r == 0 ? (uint32_t)H * wpr * 4 : (uint32_t)H * G * 2;
      if (base && !(reinterpret_cast<uintptr_t>(base) & 15)) {
        const uint32_t piece = ((bytes + gridDim.x - 1) / gridDim.x + 15u) & ~15u;
        const uint32_t b0 = blockIdx.x * piece;
        if (b0 < bytes) {
          const uint32_t sz = (bytes - b0 < piece ? bytes - b0 : piece) & ~15u;
          if (sz) prefetch_l2(base + b0, sz);
        }
      }
    }
  }
  __syncthreads();
  {
    const int tiles = I / 8, n_routed = U * tiles, n_units = n_routed + (Is ? Is / 8 : 0);
    const int count = gw < n_units ? (n_units - gw + W - 1) / W : 0;
    const float* xsum = reinterpret_cast<const float*>(smem + L.xsum);
    auto rows_of = [&](int id) {
      Rows R;
      if (id < n_routed) {
        const int u = id / tiles;
        const int r0 = (id - u * tiles) * 8;
        const size_t eo = (size_t)s_ue[u] * I;
        R.w[0] = a.wg + eo * (H / 8);
        R.w[1] = a.wu + eo * (H / 8);
        R.s[0] = a.sg + eo * (H / 64);
        R.s[1] = a.su + eo * (H / 64);
        R.b[0] = a.bg ? a.bg + eo * (H / 64) : nullptr;
        R.b[1] = a.bu ? a.bu + eo * (H / 64) : nullptr;
        R.row0[0] = R.row0[1] = r0;
        R.N = I;
      } else {
        const int r0 = (id - n_routed) * 8;
        R.w[0] = a.swg;
        R.w[1] = a.swu;
        R.s[0] = a.ssg;
        R.s[1] = a.ssu;
        R.b[0] = a.sbg;
        R.b[1] = a.sbu;
        R.row0[0] = R.row0[1] = r0;
        R.N = Is;
      }
      return R;
    };
    auto tok_of = [&](int id) {  // the staged token row of column gq
      if (id < n_routed) {
        const int u = id / tiles, pb = s_ub[u], nc = s_ub[u + 1] - pb;
        return gq < nc ? s_perm[pb + gq] / k : 0;
      }
      return gq < T ? gq : 0;
    };
    auto cols_of = [&](int id) {
      const int tok = tok_of(id);
      Cols C;
      C.xb = L.x + (uint32_t)(tok * (2 * H + 16) + cq * 32);
      C.xs = xsum;
      C.xs_stride = 8;
      C.r0c = __shfl_sync(0xffffffffu, tok, (2 * cq) * 4);
      C.r1c = __shfl_sync(0xffffffffu, tok, (2 * cq + 1) * 4);
      return C;
    };
    auto epi = [&](int id, const float (&acc)[4]) {
      int pb = 0, ncols = T, r0;
      if (id < n_routed) {
        const int u = id / tiles;
        r0 = (id - u * tiles) * 8;
        pb = s_ub[u];
        ncols = s_ub[u + 1] - pb;
      } else {
        r0 = (id - n_routed) * 8;
      }
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int n = 2 * cq + cc;
        if (n < ncols) {
          const uint16_t hv = swiglu_bf16(rbf(acc[cc]), rbf(acc[2 + cc]));
          if (id < n_routed) a.hbuf[(size_t)s_perm[pb + n] * I + r0 + gq] = hv;
          else a.hsbuf[(size_t)n * Is + r0 + gq] = hv;
        }
      }
    };
    const int G = H / 64;
    stream_units<kNS2>(smem, sbase, gw, W, count, 0, (G + kKC - 1) / kKC, G, H / 8,
                       L.ring2 + (uint32_t)(warp * kNS2 * kStage), a.scale8 != 0, rows_of, cols_of, epi);
  }
  if (!grid_barrier(a.barrier, a.status, &s_ok)) return;

  // ---- phase 3: down projection + combine, CTA = tiles of 16 hidden rows
  if (blockIdx.x * 16 >= H) return;
  stage_rows<false, kThreads>(smem, L.h, reinterpret_cast<float*>(smem + L.hsum), P, a.hbuf, 0, P, I);
  if (Is) stage_rows<false, kThreads>(smem, L.hs, reinterpret_cast<float*>(smem + L.hssum), 8, a.hsbuf, 0, T, Is);
  __syncthreads();
  float* prod = reinterpret_cast<float*>(smem + L.prod);
  float* spart = reinterpret_cast<float*>(smem + L.spart);
  const uint32_t ring = L.ring3 + (uint32_t)(warp * kNS3 * kStage);
  const float* hsum = reinterpret_cast<const float*>(smem + L.hsum);
  const float* hssum = reinterpret_cast<const float*>(smem + L.hssum);
  const int GI = I / 64;
  for (int rt = blockIdx.x; rt * 16 < H; rt += gridDim.x) {
    const int r0 = rt * 16;
    {
      auto rows_of = [&](int u) {
        const size_t eo = (size_t)s_ue[u] * H;
        Rows R;
        R.w[0] = R.w[1] = a.wd + eo * (I / 8);
        R.s[0] = R.s[1] = a.sd + eo * (I / 64);
        R.b[0] = R.b[1] = a.bd ? a.bd + eo * (I / 64) : nullptr;
        R.row0[0] = r0;
        R.row0[1] = r0 + 8;
        R.N = H;
        return R;
      };
      auto cols_of = [&](int u) {
        const int pb = s_ub[u], nc = s_ub[u + 1] - pb;
        const int prow = s_perm[pb + (gq < nc ? gq : 0)];
        Cols C;
        C.xb = L.h + (uint32_t)(prow * (2 * I + 16) + cq * 32);
        C.xs = hsum;
        C.xs_stride = P;
        C.r0c = __shfl_sync(0xffffffffu, prow, (2 * cq) * 4);
        C.r1c = __shfl_sync(0xffffffffu, prow, (2 * cq + 1) * 4);
        return C;
      };
      auto epi = [&](int u, const float (&acc)[4]) {
        const int pb = s_ub[u], nc = s_ub[u + 1] - pb;
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int n = 2 * cq + cc;
          if (n < nc) {
            const int p = s_perm[pb + n];
            const float wv = bf2f(s_w[p]);
            prod[p * 16 + gq] = rbf(__fmul_rn(rbf(acc[cc]), wv));
            prod[p * 16 + gq + 8] = rbf(__fmul_rn(rbf(acc[2 + cc]), wv));
          }
        }
      };
      const int count = warp < U ? (U - warp + WARPS - 1) / WARPS : 0;
      stream_units<kNS3>(smem, sbase, warp, WARPS, count, 0, (GI + kKC - 1) / kKC, GI, I / 8, ring,
                         a.scale8 != 0, rows_of, cols_of, epi);
    }
    if (Is) {
      // the shared expert's down projection, K split over the CTA's warps (fp32 partials
      // added in warp order below)
      const int GS = Is / 64;
      const int nch = (GS + kKC - 1) / kKC;
      const int cpw = (nch + WARPS - 1) / WARPS;
      const int cb = warp * cpw, ce = cb + cpw < nch ? cb + cpw : nch;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {  // zeros for a warp with no chunks
        const int n = 2 * cq + cc;
        if (n < T) {
          spart[(warp * 8 + n) * 16 + gq] = 0.0f;
          spart[(warp * 8 + n) * 16 + gq + 8] = 0.0f;
        }
      }
      auto rows_of = [&](int) {
        Rows R;
        R.w[0] = R.w[1] = a.swd;
        R.s[0] = R.s[1] = a.ssd;
        R.b[0] = R.b[1] = a.sbd;
        R.row0[0] = r0;
        R.row0[1] = r0 + 8;
        R.N = H;
        return R;
      };
      auto cols_of = [&](int) {
        const int tok = gq < T ? gq : 0;
        Cols C;
        C.xb = L.hs + (uint32_t)(tok * (2 * Is + 16) + cq * 32);
        C.xs = hssum;
        C.xs_stride = 8;
        C.r0c = __shfl_sync(0xffffffffu, tok, (2 * cq) * 4);
        C.r1c = __shfl_sync(0xffffffffu, tok, (2 * cq + 1) * 4);
        return C;
      };
      auto epi = [&](int, const float (&acc)[4]) {
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int n = 2 * cq + cc;
          if (n < T) {
            spart[(warp * 8 + n) * 16 + gq] = acc[cc];
            spart[(warp * 8 + n) * 16 + gq + 8] = acc[2 + cc];
          }
        }
      };
      stream_units<kNS3>(smem, sbase, 0, 1, cb < ce ? 1 : 0, cb, ce, GS, Is / 8, ring, a.scale8 != 0, rows_of,
                         cols_of, epi);
    }
    __syncthreads();
    // out[t, r0 + r] = bf16(sum over j in order of bf16(y_j * w_j)) (+ gated shared, + residual)
    for (int id = tid; id < T * 16; id += kThreads) {
      const int t = id >> 4, r = id & 15;
      float sacc = 0.0f;
      for (int j = 0; j < k; ++j) sacc = __fadd_rn(sacc, prod[(t * k + j) * 16 + r]);
      uint16_t o = f2bf(sacc);
      if (Is) {
        float ys = 0.0f;
        for (int w = 0; w < WARPS; ++w) ys = __fadd_rn(ys, spart[(w * 8 + t) * 16 + r]);
        float sv = rbf(ys);
        if (a.has_gate) sv = rbf(__fmul_rn(sv, bf2f(s_gate[t])));
        o = f2bf(__fadd_rn(bf2f(o), sv));
      }
      if (a.residual) o = f2bf(__fadd_rn(bf2f(a.residual[(size_t)t * H + r0 + r]), bf2f(o)));
      a.out[(size_t)t * H + r0 + r] = o;
    }
    __syncthreads();
  }
}

int sm_count() {
  static thread_local int set_dev = -1;
  static thread_local int nsm = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nsm;
  if (dev != set_dev) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0) nsm = n;
    set_dev = dev;
  }
  return nsm;
}

// Warps per CTA: 16 when the gate/up units (the most distinct experts T tokens can select
// times 16-row tiles, plus the shared expert's) outnumber 8 warps per SM, else 8, whose
// rings hold a unit's whole K in flight. Measured on the B200 (graph-replayed blocks, L2
// flushed): T=1 Qwen3-30B-A3B 768 units 32.8 us in 8-warp CTAs against 34.8-38.9 in
// 16-warp ones, LFM2-8B-A1B 896 units 36.9 against 38.9-41.0; Qwen1.5-MoE 1408 units 51.2
// against 47.1; T=2 Qwen3 / Qwen1.5 / LFM2 49.2 / 57.3 / 49.2 against 43.0 / 51.2 / 43.0.
int decode_warps(int T, int k, int E, int I, int Is) {
  const long long units = (long long)std::min(E, T * k) * (I / 8) + (Is ? Is / 8 : 0);
  return units > 8LL * sm_count() ? 16 : 8;
}

size_t smem_for(int T, int k, int E, int H, int I, int Is, int warps) {
  const int P = T * k;
  const DSmem m = dsmem(T, P, E, H, I, Is, warps);
  if (tk_bytes(T, P, E) > m.end2 - m.tk) return 0;
  const size_t need = m.end2 > m.end3 ? m.end2 : m.end3;
  return need <= kMaxSmem ? need : 0;
}

template <int NT, int WARPS>
cudaError_t launch_t(const DecodeArgs& a, size_t smem, cudaStream_t st) {
  auto kern = decode_block_kernel<NT, WARPS>;
  static thread_local int set_dev = -1;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev != set_dev) {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    if (err != cudaSuccess) return err;
    set_dev = dev;
  }
  int per_sm = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, WARPS * 32, smem);
  if (err != cudaSuccess) return err;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)sm_count());
  cfg.blockDim = dim3(WARPS * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int WARPS>
cudaError_t launch_w(const DecodeArgs& a, size_t smem, cudaStream_t st) {
  // the router's token loop is specialised for 1, 2, 4 or 8 tokens
  if (a.T <= 1) return launch_t<1, WARPS>(a, smem, st);
  if (a.T <= 2) return launch_t<2, WARPS>(a, smem, st);
  if (a.T <= 4) return launch_t<4, WARPS>(a, smem, st);
  return launch_t<8, WARPS>(a, smem, st);
}

}  // namespace

size_t decode_smem_bytes(int T, int k, int E, int H, int I, int Is) {
  const int P = T * k;
  if (T < 1 || T > kDecodeMaxT || P > kDecodeMaxP || E < 1 || E > 512) return 0;
  // groups of 64 in pairs (the scale copies move 2 or 4 groups), whole 16-row tiles
  if (H % 128 || I % 128 || Is % 128 || H % 16) return 0;
  return smem_for(T, k, E, H, I, Is, decode_warps(T, k, E, I, Is));
}

cudaError_t launch_decode_block(const DecodeArgs& a, cudaStream_t st) {
  const size_t smem = decode_smem_bytes(a.T, a.k, a.ta.E, a.H, a.I, a.Is);
  if (!smem) return cudaErrorInvalidValue;
  return decode_warps(a.T, a.k, a.ta.E, a.I, a.Is) == 16 ? launch_w<16>(a, smem, st) : launch_w<8>(a, smem, st);
}

}  // namespace moe
