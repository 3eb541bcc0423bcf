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
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"
#include "route.cuh"

namespace moe {

namespace {

constexpr int kThreads = kDecodeWarps * 32;
constexpr int kKC = 4;                        // groups of 64 per ring chunk
constexpr int kRowBytes = kKC * 32;           // one weight row's bytes per chunk
constexpr int kSOff = 16 * kRowBytes;         // scales of a stage: [16 rows][4] bf16
constexpr int kBOff = kSOff + 16 * kKC * 2;   // biases of a stage
constexpr int kStage = kBOff + 16 * kKC * 2;  // 2304 bytes
constexpr int kNS2 = 8;                       // gate/up ring stages per warp (HBM stream)
constexpr int kNS3 = 4;                       // down ring stages per warp (from L2)
constexpr uint64_t kWaitNs = 200ull * 1000 * 1000;
constexpr size_t kMaxSmem = 224 * 1024;  // dynamic; the static arrays below take ~1.2 KB

struct DSmem {
  uint32_t x, xsum, ring2, end2, h, hsum, hs, hssum, prod, spart, ring3, end3;
};
__host__ __device__ inline uint32_t al16(uint32_t v) { return (v + 15u) & ~15u; }
// Phase 2 and phase 3 reuse the same dynamic shared memory.
__host__ __device__ inline DSmem dsmem(int T, int P, int H, int I, int Is) {
  DSmem m{};
  uint32_t o = 0;
  m.x = o;     o = al16(o + (uint32_t)T * (2 * H + 16));       // token rows, fragment order
  m.xsum = o;  o = al16(o + (uint32_t)(H / 64) * 8 * 4);       // [G_H][8] group sums
  m.ring2 = o; o = al16(o + (uint32_t)kDecodeWarps * kNS2 * kStage);
  m.end2 = o;
  o = 0;
  m.h = o;     o = al16(o + (uint32_t)P * (2 * I + 16));       // SwiGLU rows of the pairs
  m.hsum = o;  o = al16(o + (uint32_t)(I / 64) * P * 4);       // [G_I][P]
  m.hs = o;    o = al16(o + (Is ? (uint32_t)T * (2 * Is + 16) : 0u));
  m.hssum = o; o = al16(o + (Is ? (uint32_t)(Is / 64) * 8 * 4 : 0u));
  m.prod = o;  o = al16(o + (uint32_t)P * 16 * 4);             // bf16(y * w) per pair, 16 rows
  m.spart = o; o = al16(o + (Is ? (uint32_t)kDecodeWarps * 8 * 16 * 4 : 0u));
  m.ring3 = o; o = al16(o + (uint32_t)kDecodeWarps * kNS3 * kStage);
  m.end3 = o;
  return m;
}

MOE_DEV void mma_acc(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                     uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
MOE_DEV void mma_first(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                       uint32_t b1) {
  const float z = 0.0f;
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
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

// Stages nrows rows of K bf16 (row r at src + r * K, read through L2: they may have been
// written by other CTAs of this grid) into shared rows of 2K + 16 bytes in the MMA
// fragment order of the GEMV (qgemv.cu): for each group of 64 and quarter c, elements
// 16c + {0,4,8,12, 1,5,9,13, 2,6,10,14, 3,7,11,15} as bf16 pairs; and the rows' per-group
// sums into sums[g * sstride + r]. Every thread of the CTA calls it.
MOE_DEV void stage_rows(unsigned char* smem, uint32_t dst, float* sums, int sstride, const uint16_t* src, int nrows,
                        int K) {
  const int G = K >> 6;
  const int units = nrows * G * 4;
  const int rb = 2 * K + 16;
  for (int u0 = 0; u0 < units; u0 += kThreads) {  // uniform trip count (shuffles below)
    const int u = u0 + (int)threadIdx.x;
    const bool v = u < units;
    const int c = u & 3, g = (u >> 2) % G, t = (u >> 2) / G;
    uint32_t in[8];
    if (v) {
      const uint4* p = reinterpret_cast<const uint4*>(src + (size_t)t * K + g * 64 + c * 16);
      const uint4 v0 = __ldcg(p), v1 = __ldcg(p + 1);
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

// The 16 weight rows one warp streams: ring rows 0-7 are rows row0[0]..+7 of matrix 0,
// ring rows 8-15 rows row0[1]..+7 of matrix 1 (gated: gate and up rows of the same outputs;
// plain: one matrix, row0[1] = row0[0] + 8). Pointers are at the expert's base.
struct Rows {
  const uint32_t* w[2];
  const uint16_t* s[2];
  const uint16_t* b[2];
  int row0[2];
  int N, wpr, G;
};

// One warp: acc = C fragment (MMA rows gq / gq+8, columns 2cq / 2cq+1) of the 16 rows
// against the 8 staged columns over chunks [cb, ce) of 4 groups. xb: this lane's B row
// (column gq) in the staging; xs: group sums [g * xs_stride + column's row]; r0c / r1c:
// the staged rows of columns 2cq and 2cq+1. Per group: s * sum_k x(128 + q) +
// (b - 128 s) * sum_k x in fp32, the GEMV's fold.
template <int NS>
MOE_DEV void warp_unit(const Rows& R, int cb, int ce, uint32_t ring, uint32_t xb, const float* xs, int xs_stride,
                       int r0c, int r1c, bool scale8, float (&acc)[4]) {
  const int lane = threadIdx.x & 31, gq = lane >> 2, cq = lane & 3;
  const uint32_t* src[4];
  uint32_t dst[4];
  int pgl[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int q = i * 32 + lane;
    const int rr = q >> 3, part = q & 7, gl = part >> 1, half = part & 1;
    const int m = rr >> 3;
    int row = R.row0[m] + (rr & 7);
    row = row < R.N ? row : R.N - 1;
    src[i] = R.w[m] + (size_t)row * R.wpr + part * 4 + (size_t)cb * kKC * 8;
    dst[i] = rr * kRowBytes + ((gl ^ (rr & 3)) * 32) + half * 16;
    pgl[i] = gl;
  }
  const int srr = lane & 15, which = lane >> 4, sm = srr >> 3;
  int srow = R.row0[sm] + (srr & 7);
  srow = srow < R.N ? srow : R.N - 1;
  const uint16_t* sbase = which ? R.b[sm] : R.s[sm];
  const uint16_t* ssrc = sbase ? sbase + (size_t)srow * R.G + (size_t)cb * kKC : nullptr;
  const uint32_t sdst = (which ? kBOff : kSOff) + srr * (kKC * 2);
  const int nch = (R.G + kKC - 1) / kKC;
  const int tail = R.G - (nch - 1) * kKC;
  auto issue = [&](int c) {
    const uint32_t st = ring + (uint32_t)(((c - cb) % NS) * kStage);
    const bool full = c + 1 < nch || tail == kKC;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (full || pgl[i] < tail) cp_async16(st + dst[i], src[i]);
#pragma unroll
    for (int i = 0; i < 4; ++i) src[i] += kKC * 8;
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
#pragma unroll
  for (int q = 0; q < 4; ++q) acc[q] = 0.0f;
#pragma unroll
  for (int i = 0; i < NS - 1; ++i) {
    if (cb + i < ce) issue(cb + i);
    else cp_commit();
  }
  for (int c = cb; c < ce; ++c) {
    if (c + NS - 1 < ce) issue(c + NS - 1);
    else cp_commit();
    cp_wait<NS - 1>();
    __syncwarp();
    const uint32_t st = ring + (uint32_t)(((c - cb) % NS) * kStage);
    const uint2 sw0 = lds_u2(st + kSOff + gq * (kKC * 2)), sw1 = lds_u2(st + kSOff + (gq + 8) * (kKC * 2));
    const uint2 bw0 = lds_u2(st + kBOff + gq * (kKC * 2)), bw1 = lds_u2(st + kBOff + (gq + 8) * (kKC * 2));
#pragma unroll
    for (int gl = 0; gl < kKC; ++gl) {
      const int g = c * kKC + gl;
      if (g < R.G) {
        const uint4 v0 = lds_u4(xb + g * 128), v1 = lds_u4(xb + g * 128 + 16);
        const uint32_t bfr[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        const float X0 = xs[g * xs_stride + r0c], X1 = xs[g * xs_stride + r1c];
        const uint32_t off = ((gl ^ (gq & 3)) * 32) + cq * 8;
        const uint2 wlo = lds_u2(st + gq * kRowBytes + off);
        const uint2 whi = lds_u2(st + (gq + 8) * kRowBytes + off);
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
  }
  cp_wait<0>();
  __syncwarp();
}

template <int PL>
__global__ void __launch_bounds__(kThreads, 1) decode_block_kernel(DecodeArgs a) {
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
  const int gw = blockIdx.x * kDecodeWarps + warp, W = gridDim.x * kDecodeWarps;
  const int T = a.T, k = a.k, P = T * k, H = a.H, I = a.I, Is = a.Is;
  const uint32_t sbase = (uint32_t)__cvta_generic_to_shared(smem);
  const DSmem L = dsmem(T, P, H, I, Is);

  // ---- phase 1: router logits, one row per warp
  for (int row = gw; row < a.ra.n_rows; row += W) router_tile<1, kDecodeMaxT>(a.ra, row, 0, lane);
  if (!grid_barrier(a.barrier, a.status, &s_ok)) return;

  // ---- every CTA: top-k of each token, then the grouping of the pairs by expert
  {
    TopkArgs ta = a.ta;
    ta.idx = s_idx;
    ta.weights = s_w;
    ta.packed = nullptr;
    ta.gate_val = a.has_gate ? s_gate : nullptr;
    if (warp < T) topk_token<PL>(ta, warp, lane);
  }
  __syncthreads();
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
    }
  }
  __syncthreads();
  const int U = s_U;

  // ---- phase 2: gate/up + SwiGLU of the selected experts and the shared expert
  stage_rows(smem, L.x, reinterpret_cast<float*>(smem + L.xsum), 8, a.ra.x, T, H);
  if (tid == 0) {
    // this CTA's slice of every selected expert's down weights (and the shared down)
    // into L2, so the down projection after the next barrier reads L2, not HBM
    const int wprI = I / 8, GI = I / 64;
    for (int u = 0; u <= U; ++u) {
      const bool sh = u == U;
      if (sh && !Is) break;
      const int e = sh ? 0 : s_ue[u];
      const int wpr = sh ? Is / 8 : wprI, G = sh ? Is / 64 : GI;
      const char* regions[3] = {
          reinterpret_cast<const char*>((sh ? a.swd : a.wd) + (size_t)e * H * wpr),
          reinterpret_cast<const char*>((sh ? a.ssd : a.sd) + (size_t)e * H * G),
          (sh ? a.sbd : a.bd) ? reinterpret_cast<const char*>((sh ? a.sbd : a.bd) + (size_t)e * H * G) : nullptr};
      const size_t bytes[3] = {(size_t)H * wpr * 4, (size_t)H * G * 2, (size_t)H * G * 2};
      for (int r = 0; r < 3; ++r) {
        if (!regions[r] || (reinterpret_cast<uintptr_t>(regions[r]) & 15)) continue;
        const size_t piece = ((bytes[r] + gridDim.x - 1) / gridDim.x + 15) & ~size_t(15);
        const size_t b0 = (size_t)blockIdx.x * piece;
        if (b0 >= bytes[r]) continue;
        size_t sz = bytes[r] - b0 < piece ? bytes[r] - b0 : piece;
        sz &= ~size_t(15);
        if (sz) prefetch_l2(regions[r] + b0, (uint32_t)sz);
      }
    }
  }
  __syncthreads();
  {
    const int tiles = I / 8, n_routed = U * tiles, n_units = n_routed + (Is ? Is / 8 : 0);
    const uint32_t ring = sbase + L.ring2 + (uint32_t)(warp * kNS2 * kStage);
    const float* xsum = reinterpret_cast<const float*>(smem + L.xsum);
    const int nch = (H / 64 + kKC - 1) / kKC;
    for (int id = gw; id < n_units; id += W) {
      Rows R;
      int ncols, pb = 0, r0;
      int tok;  // the staged token row of column gq
      if (id < n_routed) {
        const int u = id / tiles;
        r0 = (id - u * tiles) * 8;
        const int e = s_ue[u];
        pb = s_ub[u];
        ncols = s_ub[u + 1] - pb;
        const size_t eo = (size_t)e * I;
        R.w[0] = a.wg + eo * (H / 8);
        R.w[1] = a.wu + eo * (H / 8);
        R.s[0] = a.sg + eo * (H / 64);
        R.s[1] = a.su + eo * (H / 64);
        R.b[0] = a.bg ? a.bg + eo * (H / 64) : nullptr;
        R.b[1] = a.bu ? a.bu + eo * (H / 64) : nullptr;
        R.N = I;
        tok = gq < ncols ? s_perm[pb + gq] / k : 0;
      } else {
        r0 = (id - n_routed) * 8;
        ncols = T;
        R.w[0] = a.swg;
        R.w[1] = a.swu;
        R.s[0] = a.ssg;
        R.s[1] = a.ssu;
        R.b[0] = a.sbg;
        R.b[1] = a.sbu;
        R.N = Is;
        tok = gq < T ? gq : 0;
      }
      R.row0[0] = r0;
      R.row0[1] = r0;
      R.wpr = H / 8;
      R.G = H / 64;
      const int t0 = __shfl_sync(0xffffffffu, tok, (2 * cq) * 4);
      const int t1 = __shfl_sync(0xffffffffu, tok, (2 * cq + 1) * 4);
      const uint32_t xb = sbase + L.x + (uint32_t)(tok * (2 * H + 16) + cq * 32);
      float acc[4];
      warp_unit<kNS2>(R, 0, nch, ring, xb, xsum, 8, t0, t1, a.scale8 != 0, acc);
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int n = 2 * cq + cc;
        if (n < ncols) {
          const uint16_t hv = swiglu_bf16(rbf(acc[cc]), rbf(acc[2 + cc]));
          if (id < n_routed) a.hbuf[(size_t)s_perm[pb + n] * I + r0 + gq] = hv;
          else a.hsbuf[(size_t)n * Is + r0 + gq] = hv;
        }
      }
    }
  }
  if (!grid_barrier(a.barrier, a.status, &s_ok)) return;

  // ---- phase 3: down projection + combine, CTA = tiles of 16 hidden rows
  if (blockIdx.x * 16 >= H) return;
  stage_rows(smem, L.h, reinterpret_cast<float*>(smem + L.hsum), P, a.hbuf, P, I);
  if (Is) stage_rows(smem, L.hs, reinterpret_cast<float*>(smem + L.hssum), 8, a.hsbuf, T, Is);
  __syncthreads();
  float* prod = reinterpret_cast<float*>(smem + L.prod);
  float* spart = reinterpret_cast<float*>(smem + L.spart);
  const uint32_t ring = sbase + L.ring3 + (uint32_t)(warp * kNS3 * kStage);
  const int nchI = (I / 64 + kKC - 1) / kKC;
  for (int rt = blockIdx.x; rt * 16 < H; rt += gridDim.x) {
    const int r0 = rt * 16;
    for (int u = warp; u < U; u += kDecodeWarps) {
      const int e = s_ue[u], pb = s_ub[u], ncols = s_ub[u + 1] - pb;
      const size_t eo = (size_t)e * H;
      Rows R;
      R.w[0] = R.w[1] = a.wd + eo * (I / 8);
      R.s[0] = R.s[1] = a.sd + eo * (I / 64);
      R.b[0] = R.b[1] = a.bd ? a.bd + eo * (I / 64) : nullptr;
      R.row0[0] = r0;
      R.row0[1] = r0 + 8;
      R.N = H;
      R.wpr = I / 8;
      R.G = I / 64;
      const int prow = s_perm[pb + (gq < ncols ? gq : 0)];
      const int p0 = __shfl_sync(0xffffffffu, prow, (2 * cq) * 4);
      const int p1 = __shfl_sync(0xffffffffu, prow, (2 * cq + 1) * 4);
      const uint32_t xb = sbase + L.h + (uint32_t)(prow * (2 * I + 16) + cq * 32);
      float acc[4];
      warp_unit<kNS3>(R, 0, nchI, ring, xb, reinterpret_cast<const float*>(smem + L.hsum), P, p0, p1,
                      a.scale8 != 0, acc);
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int n = 2 * cq + cc;
        if (n < ncols) {
          const int p = s_perm[pb + n];
          const float wv = bf2f(s_w[p]);
          prod[p * 16 + gq] = rbf(__fmul_rn(rbf(acc[cc]), wv));
          prod[p * 16 + gq + 8] = rbf(__fmul_rn(rbf(acc[2 + cc]), wv));
        }
      }
    }
    if (Is) {
      // the shared expert's down projection, K split over the CTA's warps (fp32 partials
      // added in warp order below)
      Rows R;
      R.w[0] = R.w[1] = a.swd;
      R.s[0] = R.s[1] = a.ssd;
      R.b[0] = R.b[1] = a.sbd;
      R.row0[0] = r0;
      R.row0[1] = r0 + 8;
      R.N = H;
      R.wpr = Is / 8;
      R.G = Is / 64;
      const int nch = (R.G + kKC - 1) / kKC;
      const int cpw = (nch + kDecodeWarps - 1) / kDecodeWarps;
      const int cb = warp * cpw, ce = cb + cpw < nch ? cb + cpw : nch;
      const int tok = gq < T ? gq : 0;
      const int t0 = __shfl_sync(0xffffffffu, tok, (2 * cq) * 4);
      const int t1 = __shfl_sync(0xffffffffu, tok, (2 * cq + 1) * 4);
      const uint32_t xb = sbase + L.hs + (uint32_t)(tok * (2 * Is + 16) + cq * 32);
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (cb < ce)
        warp_unit<kNS3>(R, cb, ce, ring, xb, reinterpret_cast<const float*>(smem + L.hssum), 8, t0, t1,
                        a.scale8 != 0, acc);
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int n = 2 * cq + cc;
        if (n < T) {
          spart[(warp * 8 + n) * 16 + gq] = acc[cc];
          spart[(warp * 8 + n) * 16 + gq + 8] = acc[2 + cc];
        }
      }
    }
    __syncthreads();
    // out[t, r0 + r] = bf16(sum over j in order of bf16(y_j * w_j)) (+ gated shared, + residual)
    for (int id = tid; id < T * 16; id += kThreads) {
      const int t = id >> 4, r = id & 15;
      float s = 0.0f;
      for (int j = 0; j < k; ++j) s = __fadd_rn(s, prod[(t * k + j) * 16 + r]);
      uint16_t o = f2bf(s);
      if (Is) {
        float ys = 0.0f;
        for (int w = 0; w < kDecodeWarps; ++w) ys = __fadd_rn(ys, spart[(w * 8 + t) * 16 + r]);
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

template <int PL>
cudaError_t launch_t(const DecodeArgs& a, size_t smem, cudaStream_t st) {
  auto kern = decode_block_kernel<PL>;
  static thread_local int set_dev = -1;
  static thread_local int nsm = 0;
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev != set_dev) {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    if (err != cudaSuccess) return err;
    err = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    if (err != cudaSuccess) return err;
    set_dev = dev;
  }
  int per_sm = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
  if (err != cudaSuccess) return err;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)nsm);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

size_t decode_smem_bytes(int T, int k, int H, int I, int Is) {
  const int P = T * k;
  if (T < 1 || T > kDecodeMaxT || P > kDecodeMaxP) return 0;
  // groups of 64 in pairs (the scale copies move 2 or 4 groups), whole 16-row tiles
  if (H % 128 || I % 128 || Is % 128 || H % 16) return 0;
  const DSmem m = dsmem(T, P, H, I, Is);
  const size_t need = m.end2 > m.end3 ? m.end2 : m.end3;
  return need <= kMaxSmem ? need : 0;
}

cudaError_t launch_decode_block(const DecodeArgs& a, cudaStream_t st) {
  const size_t smem = decode_smem_bytes(a.T, a.k, a.H, a.I, a.Is);
  if (!smem) return cudaErrorInvalidValue;
  const int pl = (a.ta.E + 31) / 32;
  if (pl <= 1) return launch_t<1>(a, smem, st);
  if (pl <= 2) return launch_t<2>(a, smem, st);
  if (pl <= 4) return launch_t<4>(a, smem, st);
  if (pl <= 8) return launch_t<8>(a, smem, st);
  return launch_t<16>(a, smem, st);
}

}  // namespace moe
