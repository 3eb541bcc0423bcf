// qgemv.cu — grouped 4-bit GEMV/GEMM for the decode regime (few rows per expert).
//
// Replaces gather_qmm / quantized_matmul (crates/mlx-core/src/ops.rs:592-637, 830-891)
// for the SwitchGLU gate/up/down projections (qwen3_moe_python_port.rs:311-359) and the
// shared expert (:385-390) when each expert sees few tokens.
//
// One warp = one work unit = (expert, MT m16 tiles of weight rows) over the whole K and
// all of the expert's tokens (in chunks of 8*NT8). Weights stream from HBM into registers (ld.global.nc,
// 8 bytes = 16 nibbles per lane per row per group of 64) through a ring of kPF groups
// kept in flight. The expert's token rows are staged once per CTA in shared memory
// (cp.async); the 4 warps of a CTA work on the same expert. The int4 fields become bf16 pairs
// holding 128 + q with one LOP3 per pair (exact) and feed mma.sync.m16n8k16 with the
// weight rows as the M side and tokens as the N side. Each group of 64 is accumulated
// separately and folded in fp32:
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
// 16c+8+j, 16c+12+j; the lane permutes its 16 activation elements the same way with
// byte permutes, which gives the B fragment of token g.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace moe {

namespace {

constexpr int kWarps = 4;

MOE_DEV void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                            uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bf16 pair (128 + q_j, 128 + q_{j+4}) from nibbles j and j+4 of w.
MOE_DEV uint32_t nib_pair(uint32_t w, int j) {
  uint32_t r;
  const uint32_t v = w >> (4 * j);
  asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(r) : "r"(v), "r"(0x000f000fu), "r"(0x43004300u));
  return r;
}

MOE_DEV uint2 ldg_nc_u2(const uint32_t* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

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

MOE_DEV uint4 lds_u4(const uint16_t* p) {
  uint4 v;
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(p);
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}

}  // namespace

// Shared memory: [x tile: 8*NT8 token rows x (K + 8) bf16][per-warp weight rings].
// A warp's ring holds kStages chunks of kKC groups for its MT*16 weight rows; a row's
// kKC groups (kKC*32 bytes, contiguous in global memory) are copied with 16-byte
// cp.async and stored at a row stride of kKC*32 + 32 bytes, which makes the lanes'
// 8-byte fragment reads conflict-free.
template <int MT>
struct Ring {
  static constexpr int kKC = 4;                    // groups per chunk
  static constexpr int kStages = 3;                // chunks in flight + being read
  static constexpr int kRowBytes = kKC * 32 + 32;  // padded row stride
  static constexpr int kRows = MT * 16;
  static constexpr int kStageBytes = kRows * kRowBytes;
  static constexpr int kWarpBytes = kStages * kStageBytes;
};

template <bool GATED, int MT, int NT8>
__global__ void __launch_bounds__(128) qgemv_kernel(QgemvArgs a, int units_per_expert, int ctas_per_expert,
                                                    int max_slots) {
  using R = Ring<MT>;
  constexpr int ROWS = GATED ? 8 * MT : 16 * MT;  // output rows per unit
  extern __shared__ __align__(16) unsigned char smem[];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, cq = lane & 3;
  const int slot = blockIdx.x / ctas_per_expert;
  const int ut = (blockIdx.x - slot * ctas_per_expert) * 4 + warp;
  if (slot >= max_slots) return;
  if (a.n_active && slot >= *a.n_active) return;
  const int e = a.active ? a.active[slot] : slot;
  const int64_t row_begin = a.offsets ? a.offsets[e] : 0;
  const int64_t row_end = a.offsets ? a.offsets[e + 1] : a.n_identity;
  if (row_end <= row_begin) return;
  const int K = a.K, N = a.N, G = K >> 6, wpr = K >> 3;
  const int r0 = ut * ROWS;
  const bool unit_live = ut < units_per_expert && r0 < N;  // warp-uniform; the warp still stages
  const RowMap rm{a.x_mode, a.x_repeat, a.lhs, a.perm};
  const int xs_stride = K + 8;  // elements
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem);
  unsigned char* ring = smem + (size_t)8 * NT8 * xs_stride * 2 + (size_t)warp * R::kWarpBytes;
  const uint32_t ring_s = (uint32_t)__cvta_generic_to_shared(ring);

  // ring row -> global row (gated: ring rows 0-7 of a tile are gate rows, 8-15 up rows)
  auto grow = [&](int rr, const uint32_t*& W, bool& ok) -> size_t {
    const int t = rr >> 4, r = rr & 15;
    int row;
    if (GATED) {
      row = r0 + 8 * t + (r & 7);
      W = (r < 8) ? a.w0 : a.w1;
    } else {
      row = r0 + 16 * t + r;
      W = a.w0;
    }
    ok = row < N;
    return (size_t)e * N + (ok ? row : 0);
  };
  // issue the cp.async copies of chunk c into ring stage c % kStages
  auto issue_chunk = [&](int c) {
    const int g0 = c * R::kKC;
    const int ng = min(R::kKC, G - g0);
    const uint32_t st = ring_s + (uint32_t)((c % R::kStages) * R::kStageBytes);
#pragma unroll
    for (int i = 0; i < MT * R::kKC; ++i) {
      const int q = i * 32 + lane;           // 16-byte piece of the stage
      const int rr = q / (2 * R::kKC);       // ring row
      const int part = q - rr * 2 * R::kKC;  // piece within the row's kKC groups
      if ((part >> 1) < ng) {
        const uint32_t* W;
        bool ok;
        const size_t row = grow(rr, W, ok);
        if (ok) {
          const uint32_t* src = W + row * wpr + (size_t)g0 * 8 + part * 4;
          const uint32_t dst = st + rr * R::kRowBytes + part * 16;
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
        }
      }
    }
    asm volatile("cp.async.commit_group;\n" ::: "memory");
  };

  // lane's scale rows per tile: lo = MMA row gq, hi = MMA row gq + 8
  const uint16_t* slo[MT];
  const uint16_t* blo[MT];
  const uint16_t* shi[MT];
  const uint16_t* bhi[MT];
  bool oklo[MT], okhi[MT];
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const uint32_t* W;
    const size_t ol = grow(t * 16 + gq, W, oklo[t]);
    const size_t oh = grow(t * 16 + gq + 8, W, okhi[t]);
    const uint16_t* Sl = a.s0;
    const uint16_t* Bl = a.b0;
    const uint16_t* Sh = GATED ? a.s1 : a.s0;
    const uint16_t* Bh = GATED ? a.b1 : a.b0;
    slo[t] = Sl + ol * G;
    shi[t] = Sh + oh * G;
    blo[t] = Bl ? Bl + ol * G : nullptr;
    bhi[t] = Bh ? Bh + oh * G : nullptr;
  }
  const int nchunks = (G + R::kKC - 1) / R::kKC;

  for (int64_t cbase = row_begin; cbase < row_end; cbase += 8 * NT8) {
    const int ntok = (row_end - cbase < 8 * NT8) ? (int)(row_end - cbase) : 8 * NT8;
    const bool n1_live = NT8 > 1 && ntok > 8;
    // ---- weight ring prologue (its latency overlaps the activation staging)
    if (unit_live) {
#pragma unroll
      for (int c = 0; c < R::kStages - 1; ++c) {
        if (c < nchunks) issue_chunk(c);
        else asm volatile("cp.async.commit_group;\n" ::: "memory");
      }
    }
    // ---- stage the chunk's token rows (cp.async, 16 bytes per copy)
    __syncthreads();  // the previous chunk's readers are done
    {
      const int cpr = K >> 3;  // 16-byte pieces per row
      for (int idx = tid; idx < ntok * cpr; idx += 128) {
        const int t = idx / cpr, c = idx - t * cpr;
        const uint16_t* src = a.x + (size_t)rm.xrow(cbase + t) * K + c * 8;
        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(xs + (size_t)t * xs_stride + c * 8);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
      }
      asm volatile("cp.async.commit_group;\n" ::: "memory");
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    __syncthreads();
    if (!unit_live) continue;
    const uint16_t* xp[NT8];
    bool xv[NT8];
#pragma unroll
    for (int n = 0; n < NT8; ++n) {
      const int t = n * 8 + gq;
      xv[n] = t < ntok;
      xp[n] = xs + (size_t)(xv[n] ? t : 0) * xs_stride + 16 * cq;
    }
    // The staging wait above drained the ring prologue too; re-establish the ring.
    float acc[MT][NT8][4];
#pragma unroll
    for (int t = 0; t < MT; ++t)
#pragma unroll
      for (int n = 0; n < NT8; ++n)
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[t][n][q] = 0.0f;

    for (int c = 0; c < nchunks; ++c) {
      // chunk c is complete when at most kStages-2 newer groups are pending
      asm volatile("cp.async.wait_group %0;\n" ::"n"(R::kStages - 2) : "memory");
      __syncwarp();
      const unsigned char* st = ring + (c % R::kStages) * R::kStageBytes;
#pragma unroll
      for (int gl = 0; gl < R::kKC; ++gl) {
        const int g = c * R::kKC + gl;
        if (g < G) {
          uint32_t bf[NT8][8];
          float X0[NT8], X1[NT8];
#pragma unroll
          for (int n = 0; n < NT8; ++n) {
            uint32_t in[8];
            if (xv[n] && (n == 0 || n1_live)) {
              const uint4 v0 = lds_u4(xp[n] + g * 64), v1 = lds_u4(xp[n] + g * 64 + 8);
              in[0] = v0.x; in[1] = v0.y; in[2] = v0.z; in[3] = v0.w;
              in[4] = v1.x; in[5] = v1.y; in[6] = v1.z; in[7] = v1.w;
            } else {
#pragma unroll
              for (int q = 0; q < 8; ++q) in[q] = 0u;
            }
            float ps = 0.0f;
#pragma unroll
            for (int q = 0; q < 8; ++q) ps = __fadd_rn(__fadd_rn(ps, bf_lo(in[q])), bf_hi(in[q]));
            ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, 1));
            ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, 2));
            X0[n] = __shfl_sync(0xffffffffu, ps, 8 * cq);      // token n*8 + 2cq
            X1[n] = __shfl_sync(0xffffffffu, ps, 8 * cq + 4);  // token n*8 + 2cq + 1
            bf[n][0] = __byte_perm(in[0], in[2], 0x5410);  // j=0: (e0, e4)
            bf[n][1] = __byte_perm(in[4], in[6], 0x5410);  //      (e8, e12)
            bf[n][2] = __byte_perm(in[0], in[2], 0x7632);  // j=1: (e1, e5)
            bf[n][3] = __byte_perm(in[4], in[6], 0x7632);  //      (e9, e13)
            bf[n][4] = __byte_perm(in[1], in[3], 0x5410);  // j=2: (e2, e6)
            bf[n][5] = __byte_perm(in[5], in[7], 0x5410);  //      (e10, e14)
            bf[n][6] = __byte_perm(in[1], in[3], 0x7632);  // j=3: (e3, e7)
            bf[n][7] = __byte_perm(in[5], in[7], 0x7632);  //      (e11, e15)
          }
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            const float s_l = oklo[t] ? bf2f(slo[t][g]) : 0.0f;
            const float s_h = okhi[t] ? bf2f(shi[t][g]) : 0.0f;
            const float c_l = __fmaf_rn(-128.0f, s_l, (oklo[t] && blo[t]) ? bf2f(blo[t][g]) : 0.0f);
            const float c_h = __fmaf_rn(-128.0f, s_h, (okhi[t] && bhi[t]) ? bf2f(bhi[t][g]) : 0.0f);
            const uint2 wlo = *reinterpret_cast<const uint2*>(st + (t * 16 + gq) * R::kRowBytes + gl * 32 + cq * 8);
            const uint2 whi = *reinterpret_cast<const uint2*>(st + (t * 16 + gq + 8) * R::kRowBytes + gl * 32 + cq * 8);
            float d[NT8][4];
#pragma unroll
            for (int n = 0; n < NT8; ++n)
#pragma unroll
              for (int q = 0; q < 4; ++q) d[n][q] = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t a0 = nib_pair(wlo.x, j), a1 = nib_pair(whi.x, j);
              const uint32_t a2 = nib_pair(wlo.y, j), a3 = nib_pair(whi.y, j);
#pragma unroll
              for (int n = 0; n < NT8; ++n)
                if (n == 0 || n1_live) mma_bf16_16816(d[n], a0, a1, a2, a3, bf[n][2 * j], bf[n][2 * j + 1]);
            }
#pragma unroll
            for (int n = 0; n < NT8; ++n) {
              acc[t][n][0] = __fmaf_rn(c_l, X0[n], __fmaf_rn(s_l, d[n][0], acc[t][n][0]));
              acc[t][n][1] = __fmaf_rn(c_l, X1[n], __fmaf_rn(s_l, d[n][1], acc[t][n][1]));
              acc[t][n][2] = __fmaf_rn(c_h, X0[n], __fmaf_rn(s_h, d[n][2], acc[t][n][2]));
              acc[t][n][3] = __fmaf_rn(c_h, X1[n], __fmaf_rn(s_h, d[n][3], acc[t][n][3]));
            }
          }
        }
      }
      __syncwarp();  // every lane is done with this stage before it is refilled
      if (c + R::kStages - 1 < nchunks) issue_chunk(c + R::kStages - 1);
      else asm volatile("cp.async.commit_group;\n" ::: "memory");
    }
    asm volatile("cp.async.wait_group 0;\n" ::: "memory");

    // ---- epilogue: C fragment (MMA rows gq / gq+8, tokens 2cq / 2cq+1)
#pragma unroll
    for (int n = 0; n < NT8; ++n)
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        const int tok = n * 8 + 2 * cq + cc;
        if (tok < ntok) {
          const int64_t pos = cbase + tok;
          const int64_t orow = a.out_mode == 0 ? pos : rm.orig(pos);
          uint16_t* o = a.out + (size_t)orow * N;
#pragma unroll
          for (int t = 0; t < MT; ++t) {
            if (GATED) {
              const int row = r0 + 8 * t + gq;
              if (row < N) o[row] = swiglu_bf16(rbf(acc[t][n][cc]), rbf(acc[t][n][2 + cc]));
            } else {
              const int row = r0 + 16 * t + gq;
              if (row < N) o[row] = f2bf(acc[t][n][cc]);
              if (row + 8 < N) o[row + 8] = f2bf(acc[t][n][2 + cc]);
            }
          }
        }
      }
  }
}

template <bool GATED, int MT, int NT8>
static cudaError_t launch_qgemv_t(const QgemvArgs& a, int slots, cudaStream_t st) {
  constexpr int ROWS = GATED ? 8 * MT : 16 * MT;
  const int upe = (a.N + ROWS - 1) / ROWS;
  const int cpe = (upe + 3) / 4;
  const long long blocks = (long long)cpe * slots;
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidConfiguration;
  const size_t smem = (size_t)8 * NT8 * (a.K + 8) * sizeof(uint16_t) + 4 * (size_t)Ring<MT>::kWarpBytes;
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  auto kern = qgemv_kernel<GATED, MT, NT8>;
  static thread_local int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != set_dev) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (err != cudaSuccess) return err;
    set_dev = dev;
  }
  kern<<<(unsigned)blocks, 128, smem, st>>>(a, upe, cpe, slots);
  return cudaGetLastError();
}

cudaError_t launch_qgemv(const QgemvArgs& a, bool gated, int slots, int max_rows_per_expert,
                         cudaStream_t st) {
  if (slots <= 0) return cudaSuccess;
  const bool small = max_rows_per_expert <= 8;
  // Wide units (two m16 tiles per warp) amortise the activation work when there are
  // enough of them to fill the GPU; otherwise one tile per warp for parallelism.
  const int rows2 = gated ? 16 : 32;
  const bool wide = (long long)slots * ((a.N + rows2 - 1) / rows2) >= 148 * 16;
  if (gated) {
    if (wide) return small ? launch_qgemv_t<true, 2, 1>(a, slots, st) : launch_qgemv_t<true, 2, 2>(a, slots, st);
    return small ? launch_qgemv_t<true, 1, 1>(a, slots, st) : launch_qgemv_t<true, 1, 2>(a, slots, st);
  }
  if (wide) return small ? launch_qgemv_t<false, 2, 1>(a, slots, st) : launch_qgemv_t<false, 2, 2>(a, slots, st);
  return small ? launch_qgemv_t<false, 1, 1>(a, slots, st) : launch_qgemv_t<false, 1, 2>(a, slots, st);
}

}  // namespace moe
