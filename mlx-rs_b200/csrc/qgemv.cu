// qgemv.cu — grouped 4-bit GEMV/GEMM for the decode regime (few rows per expert).
//
// Replaces gather_qmm / quantized_matmul (crates/mlx-core/src/ops.rs:592-637, 830-891)
// for the SwitchGLU gate/up/down projections (qwen3_moe_python_port.rs:311-359) and the
// shared expert (:385-390) when each expert sees few tokens.
//
// Work unit = one warp = (expert, MT m16 tiles of weight rows) over the whole K, for the
// expert's tokens in chunks of 8. A CTA holds its units from the same expert, so the
// token rows are staged once per CTA: read from global memory, permuted into the MMA
// fragment order and stored in shared memory together with their per-group sums.
// Each warp streams its weight rows through its own shared-memory ring with coalesced
// 16-byte cp.async copies (a row's 4 groups = 128 contiguous bytes), NS chunks deep
// (2 for the wide units; 4 for the narrow units of small batches, where fewer warps
// share an SM and each needs more bytes in flight).
//
// Arithmetic: the int4 fields become bf16 pairs holding 128 + q with one LOP3 per pair
// (exact) and feed mma.sync.m16n8k16 with the weight rows as the M side and tokens as
// the N side. Each group of 64 is accumulated separately and folded in fp32:
//     sum_k x*(s*q + b) = s * sum_k x*(128 + q) + (b - 128*s) * sum_k x,
// so the dequantised weight is never rounded (fp32 accuracy, no per-element FMA).
//
// Gated form: an m16 tile holds 8 gate rows (MMA rows 0-7) and the same 8 up rows
// (MMA rows 8-15), so the gate and up values of one output element land in the same
// lane (C fragment c0/c2 and c1/c3) and SwiGLU runs in registers.
//
// k-permutation: lane (g = lane/4, c = lane%4) reads words 2c, 2c+1 of a group, i.e.
// elements 16c..16c+15. MMA j (j = 0..3) of a group uses the nibble pairs (j, j+4) of
// both words, so its k-slots 2c, 2c+1, 2c+8, 2c+9 hold elements 16c+j, 16c+j+4,
// 16c+8+j, 16c+12+j. The staged token rows are stored in exactly that order, so a
// lane's B fragments for a group are two 16-byte shared loads.
#include <algorithm>
#include <cmath>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace moe {

namespace {

constexpr int kKC = 4;      // groups per ring chunk (128 bytes of a weight row)
constexpr int kTok = 8;     // tokens per chunk (the MMA N)

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

// bf16 pair (128 + q_j, 128 + q_{j+4}) from nibbles j and j+4 of w.
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
MOE_DEV float2 lds_f2(uint32_t a) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];\n" : "=f"(v.x), "=f"(v.y) : "r"(a));
  return v;
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

// u8 x s8 -> s32 MMA, k = 32 per instruction.
MOE_DEV void imma(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1,
                  bool first) {
  if (first) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};\n"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
}
MOE_DEV float i2f(int v) { return (float)v; }

// Piece swizzle of the whole-K scale regions (16-byte pieces within a row).
MOE_DEV int fk_swz(int r, int G) { return (G & 31) == 0 ? ((r >> 1) & 3) : 0; }

struct RowMap {
  int x_mode, x_repeat;
  const uint32_t* lhs;
  const uint32_t* perm;
  MOE_DEV int64_t orig(int64_t pos) const { return perm ? (int64_t)perm[pos] : pos; }
  MOE_DEV int64_t xrow(int64_t pos) const {
    if (x_mode == 0) return pos;
    const int64_t i = orig(pos);
    return x_mode == 1 ? i / x_repeat : (int64_t)lhs[i];
  }
};

}  // namespace

// Shared memory:
//   xperm [kTok][(K + 8) bf16]   staged token rows in fragment order (16-byte row pad)
//   xsum  [G][kTok] fp32         per-token sums of each group of 64
//   rings [warps][NS] stages of: [MT*16 rows][128 B] weight chunk; the 32-byte group
//         slot of ring row r is stored at slot (group ^ (r & 3)), which keeps the lanes'
//         8-byte fragment reads conflict-free; then [MT*16 rows][4] bf16 scales and
//         [MT*16 rows][4] bf16 biases of the chunk's groups (copied with the weights, so
//         no scale load is outstanding in registers across a chunk).
// FK (whole-K scales; 16-warp CTAs for long K, 8-warp below): the stages hold weights
// only; each warp's scales and biases for all of K sit in one region per warp, copied
// once per CTA with coalesced 16-byte cp.async (the unit's rows are contiguous in the
// MLX layout), so every 32-byte sector of the scale arrays is fetched once instead of
// once per chunk:
//   sregion [warps][s: ring rows][G] bf16, [b: ring rows][G] bf16 (gated: the MT*8 gate
//           rows, then the MT*8 up rows), between xsum and the rings.
template <bool GATED, int MT, int NC, int NS, bool SPLIT, bool FK = false>
__global__ void __launch_bounds__(FK ? 512 : 256) qgemv_kernel(QgemvArgs a, int units_per_expert,
                                                               int ctas_per_expert, int max_slots) {
  constexpr int ROWS = GATED ? 8 * MT : 16 * MT;  // output rows per unit
  constexpr int TOK = kTok * NC;                  // tokens per pass over the weights
  constexpr int kRingRows = MT * 16;
  constexpr int kSOff = kRingRows * kKC * 32;          // scales within a stage
  constexpr int kBOff = kSOff + kRingRows * kKC * 2;     // biases within a stage
  constexpr int kStageBytes = FK ? kSOff : kBOff + kRingRows * kKC * 2;
  constexpr int kPieces = kRingRows * kKC * 2 / 32;  // 16-byte copies per lane per chunk
  constexpr int kSPieces = (2 * kRingRows + 31) / 32;  // (row, scales|biases) copies per lane
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int gq = lane >> 2, cq = lane & 3;
  // blockIdx.x = (slot * ksplit + ks) * ctas_per_expert + cta within the expert
  const int ksplit = SPLIT ? a.ksplit : 1;
  const int slot = blockIdx.x / (ctas_per_expert * ksplit);
  const int rem = blockIdx.x - slot * ctas_per_expert * ksplit;
  const int ks = SPLIT ? rem / ctas_per_expert : 0;
  const int ut = (rem - ks * ctas_per_expert) * nwarps + warp;
  pdl_wait();
  if (slot >= max_slots) return;
  if (a.n_active && slot >= *a.n_active) return;
  const int e = a.active ? a.active[slot] : slot;
  const int64_t row_begin = a.offsets ? a.offsets[e] : 0;
  const int64_t row_end = a.offsets ? a.offsets[e + 1] : a.n_identity;
  if (row_end <= row_begin) return;
  if (a.max_expert_rows && row_end - row_begin >= a.max_expert_rows) return;  // the tensor-core kernel's
  const int K = a.K, N = a.N, G = K >> 6, wpr = K >> 3;
  const int r0 = ut * ROWS;
  const bool unit_live = ut < units_per_expert && r0 < N;  // warp-uniform; the warp still stages
  const RowMap rm{a.x_mode, a.x_repeat, a.lhs, a.perm};

  const int xrow_bytes = 2 * K + 16;
  const uint32_t smem_s = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t xperm_s = smem_s;
  const uint32_t xsum_s = xperm_s + TOK * xrow_bytes;
  float* xsum = reinterpret_cast<float*>(smem + TOK * xrow_bytes);
  const uint32_t sreg_all = xsum_s + G * TOK * 4;                 // FK scale regions
  const uint32_t sreg_s = sreg_all + (uint32_t)(warp * kRingRows * G * 4);
  const uint32_t ring_s = sreg_all + (FK ? (uint32_t)(nwarps * kRingRows * G * 4) : 0u) +
                          (uint32_t)(warp * NS * kStageBytes);

  // ring row -> global weight row (clamped into the matrix: rows past N compute junk
  // that is never stored)
  auto wrow = [&](int rr) -> const uint32_t* {
    const int t = rr >> 4, r = rr & 15;
    int row;
    const uint32_t* W;
    if (GATED) {
      row = r0 + 8 * t + (r & 7);
      W = (r < 8) ? a.w0 : a.w1;
    } else {
      row = r0 + 16 * t + r;
      W = a.w0;
    }
    row = row < N ? row : N - 1;
    return W + ((size_t)e * N + row) * wpr;
  };

  // per-lane cp.async sources (advanced by one chunk per issue) and swizzled destinations
  const uint32_t* src[kPieces];
  uint32_t dst[kPieces];
  int pgl[kPieces];
#pragma unroll
  for (int i = 0; i < kPieces; ++i) {
    const int q = i * 32 + lane;
    const int rr = q >> 3, part = q & 7, gl = part >> 1, half = part & 1;
    src[i] = wrow(rr) + part * 4;
    dst[i] = rr * (kKC * 32) + ((gl ^ (rr & 3)) * 32) + half * 16;
    pgl[i] = gl;
  }
  const int nchunks = (G + kKC - 1) / kKC;
  const int tail_groups = G - (nchunks - 1) * kKC;  // groups in the last chunk
  // split-K: this CTA covers chunks [c_begin, c_end) of K (the host makes every split
  // non-empty); sources start at c_begin
  const int cpk = SPLIT ? (nchunks + ksplit - 1) / ksplit : nchunks;
  const int c_begin = SPLIT ? ks * cpk : 0;
  const int c_end = SPLIT ? ((c_begin + cpk < nchunks) ? c_begin + cpk : nchunks) : nchunks;
  const int g_begin = SPLIT ? c_begin * kKC : 0;
  const int g_end = SPLIT ? ((c_end * kKC < G) ? c_end * kKC : G) : G;
  if (SPLIT) {
#pragma unroll
    for (int i = 0; i < kPieces; ++i) src[i] += (size_t)c_begin * kKC * 8;
  }
  int issued = 0;  // chunks issued so far in this token chunk
  // Without FK, scales and biases travel with the weights into the stage: 8-byte
  // cp.async when G % 4 == 0 and the bases are 8-byte aligned, two 4-byte ones when G is
  // even and they are 4-byte aligned, otherwise plain loads and shared stores at issue
  // time (odd G, or no biases: zeros).
  const uintptr_t align_bits = reinterpret_cast<uintptr_t>(a.s0) | reinterpret_cast<uintptr_t>(a.b0) |
                               (GATED ? (reinterpret_cast<uintptr_t>(a.s1) | reinterpret_cast<uintptr_t>(a.b1)) : 0);
  const bool has_b = a.b0 != nullptr && (!GATED || a.b1 != nullptr);
  const bool s4 = has_b && (G & 1) == 0 && (align_bits & 3) == 0;
  const bool s8 = s4 && (G & 3) == 0 && (align_bits & 7) == 0;
  // ring row -> scale (which = 0) or bias (which = 1) row pointer
  auto srow = [&](int rr, int which) -> const uint16_t* {
    const int t = rr >> 4, r = rr & 15;
    int row;
    const uint16_t* S;
    if (GATED) {
      row = r0 + 8 * t + (r & 7);
      S = (r < 8) ? (which ? a.b0 : a.s0) : (which ? a.b1 : a.s1);
    } else {
      row = r0 + 16 * t + r;
      S = which ? a.b0 : a.s0;
    }
    row = row < N ? row : N - 1;
    return S ? S + ((size_t)e * N + row) * G : nullptr;
  };
  const uint16_t* ssrc[kSPieces];
  uint32_t sdst[kSPieces];
  bool sval[kSPieces];
#pragma unroll
  for (int i = 0; i < kSPieces; ++i) {
    const int q = i * 32 + lane;
    sval[i] = !FK && q < 2 * kRingRows;
    const int rr = q % kRingRows, which = q / kRingRows;
    ssrc[i] = sval[i] ? srow(rr, which) : nullptr;  // null: no biases
    sdst[i] = (which ? kBOff : kSOff) + rr * (kKC * 2);
  }
  if (SPLIT) {
#pragma unroll
    for (int i = 0; i < kSPieces; ++i)
      if (ssrc[i]) ssrc[i] += (size_t)c_begin * kKC;
  }
  auto issue_chunk = [&](int c) {
    const uint32_t st = ring_s + (uint32_t)((c % NS) * kStageBytes);
    const bool full = c + 1 < nchunks || tail_groups == kKC;
    if (full) {
#pragma unroll
      for (int i = 0; i < kPieces; ++i) cp_async16(st + dst[i], src[i]);
    } else {
#pragma unroll
      for (int i = 0; i < kPieces; ++i)
        if (pgl[i] < tail_groups) cp_async16(st + dst[i], src[i]);
    }
#pragma unroll
    for (int i = 0; i < kPieces; ++i) src[i] += kKC * 8;
#pragma unroll
    for (int i = 0; i < kSPieces; ++i) {
      if (sval[i]) {
        if (s8) {
          cp_async8(st + sdst[i], ssrc[i]);
        } else if (s4) {
          cp_async4(st + sdst[i], ssrc[i]);  // groups 0-1 of the chunk (G is even)
          if (full) cp_async4(st + sdst[i] + 4, ssrc[i] + 2);
        } else {
          uint16_t v[kKC];
#pragma unroll
          for (int q = 0; q < kKC; ++q) v[q] = (ssrc[i] && c * kKC + q < G) ? ssrc[i][q] : (uint16_t)0;
          sts_u2(st + sdst[i], v[0] | ((uint32_t)v[1] << 16), v[2] | ((uint32_t)v[3] << 16));
        }
        if (ssrc[i]) ssrc[i] += kKC;
      }
    }
    ++issued;
    cp_commit();
  };

  auto reset_src = [&]() {
#pragma unroll
    for (int i = 0; i < kPieces; ++i) src[i] -= (size_t)issued * kKC * 8;
#pragma unroll
    for (int i = 0; i < kSPieces; ++i)
      if (ssrc[i]) ssrc[i] -= (size_t)issued * kKC;
    issued = 0;
  };

  if (FK && unit_live) {
    // the unit's scale and bias rows for all of K: 2 (gated: 4) contiguous regions of
    // the MLX arrays; part of the first chunk's copy group
    // 16-byte piece p of region row r lands at piece p ^ fk_swz(r): with 64-byte rows
    // (G = 32) the lanes' 8-byte reads of 8 rows then fall in distinct banks; other G
    // (rows of 24, 48, 56, 80 ... bytes) are conflict-free as they are and the region is
    // copied flat
    constexpr int kRegions = GATED ? 4 : 2;
    const int rrows = GATED ? MT * 8 : MT * 16;
    const int rbytes = rrows * G * 2;
    const int npieces = G / 8;
#pragma unroll
    for (int rg = 0; rg < kRegions; ++rg) {
      const uint16_t* base = GATED ? (rg == 0 ? a.s0 : rg == 1 ? a.s1 : rg == 2 ? a.b0 : a.b1)
                                   : (rg == 0 ? a.s0 : a.b0);
      const unsigned char* srcb =
          reinterpret_cast<const unsigned char*>(base + ((size_t)e * N + r0) * G);
      const uint32_t dstb = sreg_s + (uint32_t)(rg * rbytes);
      if ((G & 31) == 0) {
        for (int idx = lane; idx < rrows * npieces; idx += 32) {
          const int r = idx / npieces, pc = idx - r * npieces;
          cp_async16(dstb + r * G * 2 + ((pc ^ fk_swz(r, G)) << 4), srcb + r * G * 2 + (pc << 4));
        }
      } else {
        for (int off = lane * 16; off < rbytes; off += 32 * 16) cp_async16(dstb + off, srcb + off);
      }
    }
  }
  for (int64_t cbase = row_begin; cbase < row_end; cbase += TOK) {
    const int ntok = (row_end - cbase < TOK) ? (int)(row_end - cbase) : TOK;
    reset_src();
    if (unit_live) {
#pragma unroll
      for (int i = 0; i < NS - 1; ++i) {
        if (c_begin + i < c_end) issue_chunk(c_begin + i);
        else cp_commit();
      }
    }
    __syncthreads();  // the previous chunk's readers of xperm/xsum are done
    // ---- stage the token rows: fragment-order permutation + per-group sums
    const int GS = g_end - g_begin;  // groups of this K split
    const int units = ntok * GS * 4;
    for (int u0 = 0; u0 < units; u0 += blockDim.x) {  // uniform trip count (shuffles below)
      const int u = u0 + tid;
      const bool uvalid = u < units;
      const int c = u & 3;
      const int g = g_begin + (u >> 2) % GS;
      const int t = (u >> 2) / GS;
      uint32_t in[8];
      if (uvalid) {
        const uint4* p = reinterpret_cast<const uint4*>(a.x + (size_t)rm.xrow(cbase + t) * K + g * 64 + c * 16);
        const uint4 v0 = p[0], v1 = p[1];
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
      if (uvalid) {
        uint4 o0, o1;
        o0.x = __byte_perm(in[0], in[2], 0x5410);  // j=0: (e0, e4)
        o0.y = __byte_perm(in[4], in[6], 0x5410);  //      (e8, e12)
        o0.z = __byte_perm(in[0], in[2], 0x7632);  // j=1: (e1, e5)
        o0.w = __byte_perm(in[4], in[6], 0x7632);  //      (e9, e13)
        o1.x = __byte_perm(in[1], in[3], 0x5410);  // j=2: (e2, e6)
        o1.y = __byte_perm(in[5], in[7], 0x5410);  //      (e10, e14)
        o1.z = __byte_perm(in[1], in[3], 0x7632);  // j=3: (e3, e7)
        o1.w = __byte_perm(in[5], in[7], 0x7632);  //      (e11, e15)
        uint4* d = reinterpret_cast<uint4*>(smem + (size_t)t * xrow_bytes + g * 128 + c * 32);
        d[0] = o0;
        d[1] = o1;
        if (c == 0) xsum[g * TOK + t] = ps;
      }
    }
    // tokens past ntok: zero sums (their MMA columns are never stored; zeros keep them finite)
    for (int i = tid; i < G * TOK; i += blockDim.x)
      if ((i % TOK) >= ntok) xsum[i] = 0.0f;
    __syncthreads();
    if (!unit_live) continue;

    const uint32_t xb = xperm_s + gq * xrow_bytes + cq * 32;  // token gq's fragment base (chunk 0)
    float acc[NC][MT][4];
#pragma unroll
    for (int n = 0; n < NC; ++n)
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[n][t][q] = 0.0f;

    for (int c = c_begin; c < c_end; ++c) {
      if (c + NS - 1 < c_end) issue_chunk(c + NS - 1);
      else cp_commit();
      const int g0 = c * kKC;
      cp_wait<NS - 1>();
      __syncwarp();
      const uint32_t st = ring_s + (uint32_t)((c % NS) * kStageBytes);
      // this chunk's scales and biases of the lane's rows: [tile][lo/hi] = 4 bf16 (groups)
      uint2 sw[MT][2], bw[MT][2];
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (FK) {
            // region row: gated h = 0 gate row 8t+gq, h = 1 up row 8t+gq (second region);
            // plain rows 16t+gq (+8)
            const int r = GATED ? t * 8 + gq : t * 16 + gq + 8 * h;  // row within its region
            const int fr = GATED ? h * (MT * 8) + r : r;
            const uint32_t so =
                sreg_s + (uint32_t)(fr * G * 2 + ((((g0 >> 3) ^ fk_swz(r, G))) << 4) + (g0 & 7) * 2);
            sw[t][h] = lds_u2(so);
            bw[t][h] = lds_u2(so + kRingRows * G * 2);
          } else {
            const int rr = t * 16 + gq + 8 * h;
            sw[t][h] = lds_u2(st + kSOff + rr * (kKC * 2));
            bw[t][h] = lds_u2(st + kBOff + rr * (kKC * 2));
          }
        }
#pragma unroll
      for (int gl = 0; gl < kKC; ++gl) {
        const int g = g0 + gl;
        if (g < G) {
          uint32_t bfr[NC][8];
          float2 X[NC];
#pragma unroll
          for (int n = 0; n < NC; ++n) {
            const uint32_t xbn = xb + n * kTok * xrow_bytes;
            const uint4 v0 = lds_u4(xbn + g * 128), v1 = lds_u4(xbn + g * 128 + 16);
            bfr[n][0] = v0.x; bfr[n][1] = v0.y; bfr[n][2] = v0.z; bfr[n][3] = v0.w;
            bfr[n][4] = v1.x; bfr[n][5] = v1.y; bfr[n][6] = v1.z; bfr[n][7] = v1.w;
            X[n] = lds_f2(xsum_s + (g * TOK + n * kTok + 2 * cq) * 4);  // tokens 2cq, 2cq+1 of chunk n
          }
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const int rr = t * 16 + gq;
            const uint32_t off = ((gl ^ (rr & 3)) * 32) + cq * 8;
            const uint2 wlo = lds_u2(st + rr * (kKC * 32) + off);
            const uint2 whi = lds_u2(st + (rr + 8) * (kKC * 32) + off);
            float d[NC][4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t a0 = nib_pair(wlo.x, j), a1 = nib_pair(whi.x, j);
              const uint32_t a2 = nib_pair(wlo.y, j), a3 = nib_pair(whi.y, j);
#pragma unroll
              for (int n = 0; n < NC; ++n) {
                if (j == 0) mma_first(d[n], a0, a1, a2, a3, bfr[n][0], bfr[n][1]);
                else mma_acc(d[n], a0, a1, a2, a3, bfr[n][2 * j], bfr[n][2 * j + 1]);
              }
            }
            const uint32_t s_lo2 = (gl >> 1) ? sw[t][0].y : sw[t][0].x;
            const uint32_t s_hi2 = (gl >> 1) ? sw[t][1].y : sw[t][1].x;
            const uint32_t b_lo2 = (gl >> 1) ? bw[t][0].y : bw[t][0].x;
            const uint32_t b_hi2 = (gl >> 1) ? bw[t][1].y : bw[t][1].x;
            const float s_l = (gl & 1) ? bf_hi(s_lo2) : bf_lo(s_lo2);
            const float s_h = (gl & 1) ? bf_hi(s_hi2) : bf_lo(s_hi2);
            const float c_l = __fmaf_rn(-128.0f, s_l, (gl & 1) ? bf_hi(b_lo2) : bf_lo(b_lo2));
            const float c_h = __fmaf_rn(-128.0f, s_h, (gl & 1) ? bf_hi(b_hi2) : bf_lo(b_hi2));
#pragma unroll
            for (int n = 0; n < NC; ++n) {
              acc[n][t][0] = __fmaf_rn(c_l, X[n].x, __fmaf_rn(s_l, d[n][0], acc[n][t][0]));
              acc[n][t][1] = __fmaf_rn(c_l, X[n].y, __fmaf_rn(s_l, d[n][1], acc[n][t][1]));
              acc[n][t][2] = __fmaf_rn(c_h, X[n].x, __fmaf_rn(s_h, d[n][2], acc[n][t][2]));
              acc[n][t][3] = __fmaf_rn(c_h, X[n].y, __fmaf_rn(s_h, d[n][3], acc[n][t][3]));
            }
          }
        }
      }
      __syncwarp();  // every lane is done with this stage before it is refilled
    }
    cp_wait<0>();
    pdl_trigger();

    // ---- epilogue: C fragment (MMA rows gq / gq+8, tokens 2cq / 2cq+1 of each chunk)
    if (SPLIT) {
      // fp32 partial sums of this K split: [ks][pos][N] (plain) or [ks][pos][gate N | up N]
      const int N2 = GATED ? 2 * N : N;
#pragma unroll
      for (int n = 0; n < NC; ++n)
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int tok = n * kTok + 2 * cq + cc;
          if (tok < ntok) {
            float* pr = a.partial + ((size_t)ks * a.part_rows + (size_t)(cbase + tok)) * N2;
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              if (GATED) {
                const int row = r0 + 8 * t + gq;
                if (row < N) {
                  pr[row] = acc[n][t][cc];
                  pr[N + row] = acc[n][t][2 + cc];
                }
              } else {
                const int row = r0 + 16 * t + gq;
                if (row < N) pr[row] = acc[n][t][cc];
                if (row + 8 < N) pr[row + 8] = acc[n][t][2 + cc];
              }
            }
          }
        }
    } else {
#pragma unroll
      for (int n = 0; n < NC; ++n)
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const int tok = n * kTok + 2 * cq + cc;
          if (tok < ntok) {
            const int64_t pos = cbase + tok;
            const int64_t orow = a.out_mode == 0 ? pos : rm.orig(pos);
            uint16_t* o = a.out + (size_t)orow * N;
#pragma unroll
            for (int t = 0; t < MT; ++t) {
              if (GATED) {
                const int row = r0 + 8 * t + gq;
                if (row < N)
                  o[row] = a.act ? gelu_mul_bf16(rbf(acc[n][t][cc]), rbf(acc[n][t][2 + cc]))
                                 : swiglu_bf16(rbf(acc[n][t][cc]), rbf(acc[n][t][2 + cc]));
              } else {
                const int row = r0 + 16 * t + gq;
                if (row < N) o[row] = f2bf(acc[n][t][cc]);
                if (row + 8 < N) o[row + 8] = f2bf(acc[n][t][2 + cc]);
              }
            }
          }
        }
    }
  }
}

// Integer path (decode, whole-K scales, MT = 2, 8 tokens per pass): weights enter the MMA
// as u8 nibbles (w & 0x0f0f0f0f even nibbles, (w >> 4) & 0x0f0f0f0f odd nibbles), tokens as
// two s8 limbs of a per-token fixed-point mantissa m = rint(x * 2^-E), |m| < 2^14,
// m = 128 * hi + lo, lo in [0, 127]. Two column chunks of 8 MMA columns; in chunk n,
// column 2t + limb holds token 4n + t (t = 0..3), so a lane's C fragment of chunk n holds
// token 4n + cq's (hi, lo) sums for rows gq and gq+8 (the weight fragments serve both):
//   sum_k x*(s*q + b) = 2^E * (s * (128*D_hi + D_lo) + b * X'),  X' = sum_k m.
// k-permutation per 32-k MMA (word 2cq for MMA 0, 2cq+1 for MMA 1 of a group): k-slots
// 4cq+i hold element 16cq + 2i (+8 for MMA 1), k-slots 16+4cq+i element 16cq + 2i + 1.
// Shared memory: xq [16 columns][K + 64 B] s8 limbs in fragment order, xs [G][8] float X',
// emax [8] int, scale regions (as FK), rings (weights only).
template <bool GATED>
__global__ void __launch_bounds__(512) qgemv_i8_kernel(QgemvArgs a, int units_per_expert, int ctas_per_expert,
                                                       int max_slots) {
  constexpr int MT = 2, NS = 2;
  constexpr int ROWS = GATED ? 8 * MT : 16 * MT;
  constexpr int TOK = 8;
  constexpr int kCols = 16;
  constexpr int kRingRows = MT * 16;
  constexpr int kStageBytes = kRingRows * kKC * 32;
  constexpr int kPieces = kRingRows * kKC * 2 / 32;
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nwarps = blockDim.x >> 5;
  const int gq = lane >> 2, cq = lane & 3;
  const int slot = blockIdx.x / ctas_per_expert;
  const int ut = (blockIdx.x - slot * ctas_per_expert) * nwarps + warp;
  pdl_wait();
  if (slot >= max_slots) return;
  if (a.n_active && slot >= *a.n_active) return;
  const int e = a.active ? a.active[slot] : slot;
  const int64_t row_begin = a.offsets ? a.offsets[e] : 0;
  const int64_t row_end = a.offsets ? a.offsets[e + 1] : a.n_identity;
  if (row_end <= row_begin) return;
  if (a.max_expert_rows && row_end - row_begin >= a.max_expert_rows) return;
  const int K = a.K, N = a.N, G = K >> 6, wpr = K >> 3;
  const int r0 = ut * ROWS;
  const bool unit_live = ut < units_per_expert && r0 < N;
  const RowMap rm{a.x_mode, a.x_repeat, a.lhs, a.perm};

  const int col_bytes = K + 64;  // 16-word column offset: conflict-free 16-byte fragment reads
  const uint32_t smem_s = (uint32_t)__cvta_generic_to_shared(smem);
  const uint32_t xq_s = smem_s;
  const uint32_t xs_s = xq_s + kCols * col_bytes;
  float* xs = reinterpret_cast<float*>(smem + kCols * col_bytes);           // [G][TOK]
  int* emax = reinterpret_cast<int*>(smem + kCols * col_bytes + G * TOK * 4);  // [TOK]
  const uint32_t sreg_all = xs_s + G * TOK * 4 + TOK * 4;  // after emax [TOK] (16-byte multiple)
  const uint32_t sreg_s = sreg_all + (uint32_t)(warp * kRingRows * G * 4);
  const uint32_t ring_s = sreg_all + (uint32_t)(nwarps * kRingRows * G * 4) + (uint32_t)(warp * NS * kStageBytes);

  auto wrow = [&](int rr) -> const uint32_t* {
    const int t = rr >> 4, r = rr & 15;
    int row;
    const uint32_t* W;
    if (GATED) {
      row = r0 + 8 * t + (r & 7);
      W = (r < 8) ? a.w0 : a.w1;
    } else {
      row = r0 + 16 * t + r;
      W = a.w0;
    }
    row = row < N ? row : N - 1;
    return W + ((size_t)e * N + row) * wpr;
  };
  const uint32_t* src[kPieces];
  uint32_t dst[kPieces];
#pragma unroll
  for (int i = 0; i < kPieces; ++i) {
    const int q = i * 32 + lane;
    const int rr = q >> 3, part = q & 7, gl = part >> 1, half = part & 1;
    src[i] = wrow(rr) + part * 4;
    dst[i] = rr * (kKC * 32) + ((gl ^ (rr & 3)) * 32) + half * 16;
  }
  const int nchunks = G / kKC;  // the launcher requires G % 4 == 0
  int issued = 0;
  auto issue_chunk = [&](int c) {
    const uint32_t st = ring_s + (uint32_t)((c % NS) * kStageBytes);
#pragma unroll
    for (int i = 0; i < kPieces; ++i) cp_async16(st + dst[i], src[i]);
#pragma unroll
    for (int i = 0; i < kPieces; ++i) src[i] += kKC * 8;
    ++issued;
    cp_commit();
  };
  auto reset_src = [&]() {
#pragma unroll
    for (int i = 0; i < kPieces; ++i) src[i] -= (size_t)issued * kKC * 8;
    issued = 0;
  };
  if (unit_live) {  // whole-K scale regions, as in qgemv_kernel's FK mode
    constexpr int kRegions = GATED ? 4 : 2;
    const int rrows = GATED ? MT * 8 : MT * 16;
    const int rbytes = rrows * G * 2;
    const int npieces = G / 8;
#pragma unroll
    for (int rg = 0; rg < kRegions; ++rg) {
      const uint16_t* base = GATED ? (rg == 0 ? a.s0 : rg == 1 ? a.s1 : rg == 2 ? a.b0 : a.b1)
                                   : (rg == 0 ? a.s0 : a.b0);
      const unsigned char* srcb = reinterpret_cast<const unsigned char*>(base + ((size_t)e * N + r0) * G);
      const uint32_t dstb = sreg_s + (uint32_t)(rg * rbytes);
      if ((G & 31) == 0) {
        for (int idx = lane; idx < rrows * npieces; idx += 32) {
          const int r = idx / npieces, pc = idx - r * npieces;
          cp_async16(dstb + r * G * 2 + ((pc ^ fk_swz(r, G)) << 4), srcb + r * G * 2 + (pc << 4));
        }
      } else {
        for (int off = lane * 16; off < rbytes; off += 32 * 16) cp_async16(dstb + off, srcb + off);
      }
    }
  }

  for (int64_t cbase = row_begin; cbase < row_end; cbase += TOK) {
    const int ntok = (row_end - cbase < TOK) ? (int)(row_end - cbase) : TOK;
    reset_src();
    if (unit_live) issue_chunk(0);
    __syncthreads();  // previous pass's readers of xq / xs / emax are done
    // ---- stage: per-token largest magnitude, then the limbs in fragment order and X'
    const int units = ntok * G * 4;
    for (int i = tid; i < TOK; i += blockDim.x) emax[i] = 0;
    __syncthreads();
    for (int u = tid; u < units; u += blockDim.x) {
      const int c = u & 3, g = (u >> 2) % G, t = (u >> 2) / G;
      const uint4* p = reinterpret_cast<const uint4*>(a.x + (size_t)rm.xrow(cbase + t) * K + g * 64 + c * 16);
      const uint4 v0 = p[0], v1 = p[1];
      const uint32_t in[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      uint32_t m = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) m = max(m, max(in[i] & 0x7fffu, (in[i] >> 16) & 0x7fffu));
      atomicMax(&emax[t], (int)m);
    }
    __syncthreads();
    for (int u0 = 0; u0 < units; u0 += blockDim.x) {  // uniform trip count (shuffles below)
      const int u = u0 + tid;
      const bool uvalid = u < units;
      const int c = u & 3, g = (u >> 2) % G, t = (u >> 2) / G;
      int mi[16];
      if (uvalid) {
        const uint4* p = reinterpret_cast<const uint4*>(a.x + (size_t)rm.xrow(cbase + t) * K + g * 64 + c * 16);
        const uint4 v0 = p[0], v1 = p[1];
        const uint32_t in[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
        // 2^-E with the row's largest |x| * 2^-E in [2^13, 2^14) (zero / non-finite rows: E = 0)
        const int mb = emax[t];
        int sh = 0;
        if (mb != 0 && mb < 0x7f80) {
          const int ex = (mb >> 7) - 127;  // floor(log2 max) for normal values
          sh = 13 - (ex < -126 ? -126 : ex);
          sh = sh > 126 ? 126 : sh;
        }
        const float sc = __int_as_float((sh + 127) << 23);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          mi[2 * i] = __float2int_rn(bf_lo(in[i]) * sc);
          mi[2 * i + 1] = __float2int_rn(bf_hi(in[i]) * sc);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) mi[i] = 0;
      }
      int xsum = 0;
#pragma unroll
      for (int i = 0; i < 16; ++i) xsum += mi[i];
      xsum += __shfl_xor_sync(0xffffffffu, xsum, 1);
      xsum += __shfl_xor_sync(0xffffffffu, xsum, 2);
      if (uvalid) {
        // column 2t: hi limbs, 2t+1: lo limbs; 16 bytes per (column, group, quarter):
        // [e0 e2 e4 e6 | e1 e3 e5 e7 | e8 e10 e12 e14 | e9 e11 e13 e15]
        auto pack = [&](int i0, int limb) -> uint32_t {
          uint32_t r = 0;
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const int m = mi[i0 + 2 * b];
            const int v = limb ? (m & 127) : (m >> 7);
            r |= ((uint32_t)v & 0xffu) << (8 * b);
          }
          return r;
        };
#pragma unroll
        for (int limb = 0; limb < 2; ++limb) {
          const uint4 o = make_uint4(pack(0, limb), pack(1, limb), pack(8, limb), pack(9, limb));
          // token t: chunk t / 4, column 2 (t % 4) + limb of the chunk
          *reinterpret_cast<uint4*>(smem + (size_t)(8 * (t >> 2) + 2 * (t & 3) + limb) * col_bytes + g * 64 + c * 16) = o;
        }
        if (c == 0) xs[g * TOK + t] = (float)xsum;
      }
    }
    for (int i = tid; i < G * TOK; i += blockDim.x)
      if ((i % TOK) >= ntok) xs[i] = 0.0f;
    __syncthreads();
    if (!unit_live) continue;

    const uint32_t xb = xq_s + gq * col_bytes + cq * 16;  // column gq's fragment base
    float acc[MT][2][2];  // [tile][chunk n: token 4n + cq][row gq / gq+8]
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int n = 0; n < 2; ++n) acc[t][n][0] = acc[t][n][1] = 0.0f;
    for (int c = 0; c < nchunks; ++c) {
      if (c + 1 < nchunks) issue_chunk(c + 1);
      else cp_commit();
      const int g0 = c * kKC;
      cp_wait<NS - 1>();
      __syncwarp();
      const uint32_t st = ring_s + (uint32_t)((c % NS) * kStageBytes);
      uint2 sw[MT][2], bw[MT][2];
#pragma unroll
      for (int t = 0; t < MT; ++t)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = GATED ? t * 8 + gq : t * 16 + gq + 8 * h;
          const int fr = GATED ? h * (MT * 8) + r : r;
          const uint32_t so = sreg_s + (uint32_t)(fr * G * 2 + ((((g0 >> 3) ^ fk_swz(r, G))) << 4) + (g0 & 7) * 2);
          sw[t][h] = lds_u2(so);
          bw[t][h] = lds_u2(so + kRingRows * G * 2);
        }
#pragma unroll
      for (int gl = 0; gl < kKC; ++gl) {
        const int g = g0 + gl;
        uint4 bf[2];  // per column chunk: (b0, b1) of MMA 0, (b0, b1) of MMA 1
        float X[2];
#pragma unroll
        for (int n = 0; n < 2; ++n) {
          bf[n] = lds_u4(xb + n * 8 * col_bytes + g * 64);
          X[n] = xs[g * TOK + 4 * n + cq];
        }
#pragma unroll
        for (int t = 0; t < MT; ++t) {
          const int rr = t * 16 + gq;
          const uint32_t off = ((gl ^ (rr & 3)) * 32) + cq * 8;
          const uint2 wlo = lds_u2(st + rr * (kKC * 32) + off);
          const uint2 whi = lds_u2(st + (rr + 8) * (kKC * 32) + off);
          const uint32_t a0 = wlo.x & 0x0f0f0f0fu, a1 = whi.x & 0x0f0f0f0fu;
          const uint32_t a2 = (wlo.x >> 4) & 0x0f0f0f0fu, a3 = (whi.x >> 4) & 0x0f0f0f0fu;
          const uint32_t a4 = wlo.y & 0x0f0f0f0fu, a5 = whi.y & 0x0f0f0f0fu;
          const uint32_t a6 = (wlo.y >> 4) & 0x0f0f0f0fu, a7 = (whi.y >> 4) & 0x0f0f0f0fu;
          const uint32_t s_lo2 = (gl >> 1) ? sw[t][0].y : sw[t][0].x;
          const uint32_t s_hi2 = (gl >> 1) ? sw[t][1].y : sw[t][1].x;
          const uint32_t b_lo2 = (gl >> 1) ? bw[t][0].y : bw[t][0].x;
          const uint32_t b_hi2 = (gl >> 1) ? bw[t][1].y : bw[t][1].x;
          const float s_l = (gl & 1) ? bf_hi(s_lo2) : bf_lo(s_lo2);
          const float s_h = (gl & 1) ? bf_hi(s_hi2) : bf_lo(s_hi2);
          const float b_l = (gl & 1) ? bf_hi(b_lo2) : bf_lo(b_lo2);
          const float b_h = (gl & 1) ? bf_hi(b_hi2) : bf_lo(b_hi2);
#pragma unroll
          for (int n = 0; n < 2; ++n) {
            int d[4];
            imma(d, a0, a1, a2, a3, bf[n].x, bf[n].y, true);
            imma(d, a4, a5, a6, a7, bf[n].z, bf[n].w, false);
            // (hi, lo) sums of token 4n + cq: c0/c1 row gq, c2/c3 row gq+8 (exact below 2^24)
            const float v_l = __fmaf_rn(128.0f, i2f(d[0]), i2f(d[1]));
            const float v_h = __fmaf_rn(128.0f, i2f(d[2]), i2f(d[3]));
            acc[t][n][0] = __fmaf_rn(b_l, X[n], __fmaf_rn(s_l, v_l, acc[t][n][0]));
            acc[t][n][1] = __fmaf_rn(b_h, X[n], __fmaf_rn(s_h, v_h, acc[t][n][1]));
          }
        }
      }
      __syncwarp();
    }
    cp_wait<0>();
    pdl_trigger();
    // ---- epilogue: tokens cq and 4 + cq, rows gq / gq+8 of each tile; undo 2^-E
#pragma unroll
    for (int n = 0; n < 2; ++n) {
    const int tok = 4 * n + cq;
    if (tok < ntok) {
      const int mb = emax[tok];
      int sh = 0;
      if (mb != 0 && mb < 0x7f80) {
        const int ex = (mb >> 7) - 127;
        sh = 13 - (ex < -126 ? -126 : ex);
        sh = sh > 126 ? 126 : sh;
      }
      // 2^-sh, sh in [-114, 126]; a token row holding inf or NaN has no fixed-point form
      // (its limbs saturated): its outputs become NaN, as the bf16 kernel's would
      const float us = mb >= 0x7f80 ? __int_as_float(0x7fc00000) : __int_as_float((127 - sh) << 23);
      const int64_t pos = cbase + tok;
      const int64_t orow = a.out_mode == 0 ? pos : rm.orig(pos);
      uint16_t* o = a.out + (size_t)orow * N;
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        if (GATED) {
          const int row = r0 + 8 * t + gq;
          if (row < N)
            o[row] = a.act ? gelu_mul_bf16(rbf(acc[t][n][0] * us), rbf(acc[t][n][1] * us))
                           : swiglu_bf16(rbf(acc[t][n][0] * us), rbf(acc[t][n][1] * us));
        } else {
          const int row = r0 + 16 * t + gq;
          if (row < N) o[row] = f2bf(acc[t][n][0] * us);
          if (row + 8 < N) o[row + 8] = f2bf(acc[t][n][1] * us);
        }
      }
    }
    }
  }
}

// Split-K reduction: out[row(pos), n] from the ksplit fp32 partials, added in split
// order, then SwiGLU (gated, the exact bf16 sequence of the GEMV epilogue) or bf16
// rounding. Rows of experts that the GEMV skipped (max_expert_rows) are left alone.
template <bool GATED>
__global__ void __launch_bounds__(256) qgemv_reduce_kernel(QgemvArgs a, int num_slots_e) {
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  pdl_trigger();
  const int N = a.N;
  if (id >= a.part_rows * N) return;
  const int64_t pos = id / N;
  const int n = (int)(id - pos * N);
  if (a.offsets) {
    const int64_t valid = a.offsets[num_slots_e];
    if (pos >= valid) return;
    if (a.max_expert_rows) {
      int l = 0, r = num_slots_e;  // expert e with offsets[e] <= pos < offsets[e + 1]
      while (r - l > 1) {
        const int m = (l + r) >> 1;
        if (a.offsets[m] <= pos) l = m;
        else r = m;
      }
      const int64_t cnt = a.offsets[l + 1] - a.offsets[l];
      if (cnt >= a.max_expert_rows) return;
    }
  }
  const int N2 = GATED ? 2 * N : N;
  float g = 0.0f, u = 0.0f;
  for (int k = 0; k < a.ksplit; ++k) {
    const float* pr = a.partial + ((size_t)k * a.part_rows + pos) * N2;
    g = __fadd_rn(g, pr[n]);
    if (GATED) u = __fadd_rn(u, pr[N + n]);
  }
  RowMap rm{a.x_mode, a.x_repeat, a.lhs, a.perm};
  const int64_t orow = a.out_mode == 0 ? pos : rm.orig(pos);
  a.out[(size_t)orow * N + n] =
      GATED ? (a.act ? gelu_mul_bf16(rbf(g), rbf(u)) : swiglu_bf16(rbf(g), rbf(u))) : f2bf(g);
}

template <int MT, int NC, int NS, bool FK>
static size_t qgemv_smem(int K, int wpc) {
  const int G = K / 64;
  return (size_t)kTok * NC * (2 * K + 16) + (size_t)G * kTok * NC * 4 +
         (FK ? (size_t)wpc * MT * 16 * G * 4 + (size_t)wpc * NS * MT * 16 * kKC * 32
             : (size_t)wpc * NS * MT * 16 * (kKC * 32 + kKC * 4));  // weights (+ scales + biases)
}

template <bool GATED, int MT, int NC, int NS, bool SPLIT, bool FK = false>
static cudaError_t launch_split_t(const QgemvArgs& a, int upe, int cpe, int slots, int wpc, cudaStream_t st) {
  const long long blocks = (long long)cpe * slots * a.ksplit;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  const size_t smem = qgemv_smem<MT, NC, NS, FK>(a.K, wpc);
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  auto kern = qgemv_kernel<GATED, MT, NC, NS, SPLIT, FK>;
  static thread_local int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != set_dev) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (err != cudaSuccess) return err;
    set_dev = dev;
  }
  return launch_k(kern, dim3((unsigned)blocks), dim3(wpc * 32), smem, st, a, upe, cpe, slots);
}

template <bool GATED, int MT, int NC, int NS, bool FK = false>
static cudaError_t launch_qgemv_t(const QgemvArgs& a0, int slots, int wpc, cudaStream_t st) {
  constexpr int ROWS = GATED ? 8 * MT : 16 * MT;
  QgemvArgs a = a0;
  const int upe = (a.N + ROWS - 1) / ROWS;
  const int cpe = (upe + wpc - 1) / wpc;
  // Split K when the units of work would leave most of the GPU idle (few experts and
  // few rows: the shared expert, or T <= a few tokens) and the partials fit the buffer.
  a.ksplit = 1;
  {
    const int nchunks = (a.K / 64 + kKC - 1) / kKC;
    const long long warps = (long long)slots * cpe * wpc;
    int ks = 1;
    // only when under an eighth of the GPU's warp slots would be busy (the Qwen1.5 shared
    // expert at T=1: 128 warps): a split adds a reduction launch and a round trip of fp32
    // partials, which measured slower already at 512 warps (LFM2 down projection, T=1)
    if (warps * 8 <= 148LL * 16)
      while (ks < 8 && warps * ks * 2 <= 148LL * 16 && 2 * ks <= nchunks) ks *= 2;
    const char* env = std::getenv("MOE_B200_SPLITK");  // "0": never split (tests compare both)
    if (ks > 1 && a.partial && a.part_rows > 0 && !(env && env[0] == '0')) {
      const int cpk = (nchunks + ks - 1) / ks;
      ks = (nchunks + cpk - 1) / cpk;  // every split non-empty
      const size_t need = (size_t)ks * a.part_rows * (GATED ? 2 : 1) * a.N * sizeof(float);
      if (ks > 1 && need <= a.partial_bytes) a.ksplit = ks;
    }
  }
  if (FK) {  // chosen only for grids that fill the GPU, which are never split
    a.ksplit = 1;
    return launch_split_t<GATED, MT, NC, NS, false, FK>(a, upe, cpe, slots, wpc, st);
  }
  cudaError_t err = a.ksplit > 1 ? launch_split_t<GATED, MT, NC, NS, true>(a, upe, cpe, slots, wpc, st)
                                  : launch_split_t<GATED, MT, NC, NS, false>(a, upe, cpe, slots, wpc, st);
  if (err != cudaSuccess || a.ksplit == 1) return err;
  const long long n = a.part_rows * (long long)a.N;
  return launch_k(qgemv_reduce_kernel<GATED>, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, a,
                  a.num_experts_total);
}

cudaError_t launch_gemv_reduce(const QgemvArgs& a, bool gated, cudaStream_t st) {
  const long long n = a.part_rows * (long long)a.N;
  if (n <= 0 || a.ksplit <= 1) return cudaSuccess;
  const dim3 grid((unsigned)((n + 255) / 256));
  return gated ? launch_k(qgemv_reduce_kernel<true>, grid, dim3(256), 0, st, a, a.num_experts_total)
               : launch_k(qgemv_reduce_kernel<false>, grid, dim3(256), 0, st, a, a.num_experts_total);
}

// Whole-K scales for the wide one-token-chunk case: warps per CTA (16 or 8) or 0 when
// not used. Needs the unit's scale rows whole, 16-byte aligned regions and 8-byte
// aligned chunk scales (G % 4 == 0). Long K (G >= 24, G % 8 == 0: 16-byte rows) runs
// 16-warp CTAs, whose one staging of x serves twice the rows and leaves room for the
// scales; shorter K keeps 8-warp CTAs, two per SM (measured: K = 2048 in 16-warp CTAs
// gains 9% and K = 768 loses 6% against per-chunk scale copies).
static int fk_warps(const QgemvArgs& a, bool gated) {
  const int G = a.K / 64;
  const int rows = gated ? 16 : 32;  // rows of one unit (MT = 2)
  const uintptr_t al = reinterpret_cast<uintptr_t>(a.s0) | reinterpret_cast<uintptr_t>(a.b0) |
                       (gated ? reinterpret_cast<uintptr_t>(a.s1) | reinterpret_cast<uintptr_t>(a.b1) : 0);
  if (!a.b0 || (gated && !a.b1) || (al & 15) || (G & 3) || (a.N % rows)) return 0;
  if (((size_t)a.N * G * 2) % 16) return 0;  // expert stride of the scale arrays
  const char* env = std::getenv("MOE_B200_GEMV_FK");  // "0": per-chunk scales only
  if (env && env[0] == '0') return 0;
  if (G >= 24 && (G & 7) == 0 && qgemv_smem<2, 1, 2, true>(a.K, 16) <= 227 * 1024) return 16;
  if (G < 24 && 2 * (qgemv_smem<2, 1, 2, true>(a.K, 8) + 1024) <= 228 * 1024) return 8;
  return 0;
}

template <bool GATED>
static cudaError_t launch_i8(const QgemvArgs& a, int slots, int wpc, cudaStream_t st) {
  constexpr int ROWS = GATED ? 16 : 32;
  const int upe = (a.N + ROWS - 1) / ROWS;
  const int cpe = (upe + wpc - 1) / wpc;
  const long long blocks = (long long)cpe * slots;
  const int G = a.K / 64;
  const size_t smem = (size_t)16 * (a.K + 64) + (size_t)G * 8 * 4 + 32 + (size_t)wpc * 32 * G * 4 +
                      (size_t)wpc * 2 * 32 * kKC * 32;
  if (smem > 227 * 1024 || blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  static thread_local int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != set_dev) {
    cudaError_t err = cudaFuncSetAttribute(qgemv_i8_kernel<GATED>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           227 * 1024);
    if (err != cudaSuccess) return err;
    set_dev = dev;
  }
  return launch_k(qgemv_i8_kernel<GATED>, dim3((unsigned)blocks), dim3(wpc * 32), smem, st, a, upe, cpe, slots);
}

template <bool GATED, int NC>
static cudaError_t launch_qgemv_nc(const QgemvArgs& a, int slots, bool wide, double active, cudaStream_t st) {
  {
    const char* env = std::getenv("MOE_B200_GEMV_I8");  // prototype: integer MMA path
    if (env && env[0] == '1' && NC == 1 && wide && (a.K / 64) % 4 == 0) {
      const int fw = fk_warps(a, GATED);
      if (fw) return launch_i8<GATED>(a, slots, fw, st);
    }
  }
  if (NC == 1 && wide) {
    const int fw = fk_warps(a, GATED);
    // Long-K gated launches (16-warp CTAs of two-tile units by default): unit size and CTA
    // shape by the expected grid (all three forms give identical bits). Measured on the
    // B200, gate/up launch of graph-replayed blocks:
    //  - the two-tile grid fills at most ~1.25 waves: one-tile units in 8-warp CTAs, two per
    //    SM (Qwen3-30B-A3B T=8 48.0 -> 42.5 us; LFM2-8B-A1B T=8 28.7 -> 22.6 us);
    //  - an expert spans 5 or more 16-warp CTAs (N >= 1280): one-tile units in 16-warp CTAs
    //    with 4-chunk rings (LFM2 T=32 / 64 / 128: 66.5 / 111.5 / 88.0 -> 56.3 / 85.0 /
    //    70.7 us);
    //  - otherwise two-tile units (Qwen3 T=32 / 64: 73.7 / 91.1 us; one-tile units took
    //    74.8-78.9 / 91.2-95.2).
    if (GATED && fw == 16) {
      const int upe2 = (a.N + 15) / 16;
      const double ctas2 = active * ((upe2 + 15) / 16);
      if (ctas2 <= 1.25 * 148 && 2 * (qgemv_smem<1, 1, 2, true>(a.K, 8) + 1024) <= 228 * 1024)
        return launch_qgemv_t<GATED, 1, 1, 2, true>(a, slots, 8, st);
      if (upe2 >= 80 && qgemv_smem<1, 1, 4, true>(a.K, 16) <= 227 * 1024)
        return launch_qgemv_t<GATED, 1, 1, 4, true>(a, slots, 16, st);
    }
    if (fw) return launch_qgemv_t<GATED, 2, 1, 2, true>(a, slots, fw, st);
  }
  return wide ? launch_qgemv_t<GATED, 2, NC, 2>(a, slots, 8, st) : launch_qgemv_t<GATED, 1, NC, 4>(a, slots, 4, st);
}

cudaError_t launch_qgemv(const QgemvArgs& a, bool gated, int slots, int rows_per_expert,
                         cudaStream_t st) {
  if (slots <= 0) return cudaSuccess;
  // Wide units (two m16 tiles per warp) and 8-warp CTAs when there is enough work to
  // fill the GPU; narrow units in 4-warp CTAs otherwise, for parallelism.
  const int rows2 = gated ? 16 : 32;
  const bool wide = (long long)slots * ((a.N + rows2 - 1) / rows2) >= 148 * 16;
  // Tokens per pass over an expert's weights: 8 up to 16 expected rows per expert, 32
  // above (an expert with more rows takes more passes), while the staged rows fit; 16 only
  // when 32 do not fit. Measured on the B200 (Qwen3-30B-A3B shapes, graph-replayed blocks):
  // up to 16 expected rows, 8-token passes of the whole-K-scale kernel beat 16-token passes
  // (T=96: 172 against 211 us; T=192: 248 against 262 us), and above 16 rows 32-token
  // passes beat 16-token ones (T=320: 341 against 365 us).
  int nc = rows_per_expert > 16 ? 4 : 1;
  while (nc > 1 && (size_t)kTok * nc * (2 * a.K + 16) > 140 * 1024) nc >>= 1;
  // expected experts with rows: slots * rows_per_expert rows spread over the experts
  const int E = a.num_experts_total > 0 ? a.num_experts_total : slots;
  const double active =
      std::min<double>(slots, E * (1.0 - std::exp(-(double)slots * rows_per_expert / E)));
  if (gated) {
    if (nc == 4) return launch_qgemv_nc<true, 4>(a, slots, wide, active, st);
    if (nc == 2) return launch_qgemv_nc<true, 2>(a, slots, wide, active, st);
    return launch_qgemv_nc<true, 1>(a, slots, wide, active, st);
  }
  if (nc == 4) return launch_qgemv_nc<false, 4>(a, slots, wide, active, st);
  if (nc == 2) return launch_qgemv_nc<false, 2>(a, slots, wide, active, st);
  return launch_qgemv_nc<false, 1>(a, slots, wide, active, st);
}

}  // namespace moe
