// qgemv.cu — grouped 4-bit GEMV/GEMM for the decode regime (few rows per expert).
//
// Replaces gather_qmm / quantized_matmul (crates/mlx-core/src/ops.rs:592-637, 830-891)
// for the SwitchGLU gate/up/down projections (qwen3_moe_python_port.rs:311-359) and the
// shared expert (:385-390) when each expert sees few tokens.
//
// Layout: one CTA = 4 warps = one expert x a tile of weight rows x a chunk of at most
// TOK (8 or 16) tokens; the 4 warps split the K groups (64 elements each) and their
// fp32 partials are summed in warp order at the end. Weights stream straight from
// HBM into registers (ld.global.nc, 8 bytes = 16 nibbles per lane per row per group),
// are turned into bf16 pairs holding 128 + q with one LOP3 per pair (exact), and feed
// mma.sync.m16n8k16 with the weight rows as the M side and tokens as the N side.
// Each group of 64 is accumulated separately and folded in fp32:
//     sum_k x*(s*q + b) = s * sum_k x*(128 + q) + (b - 128*s) * sum_k x,
// so the dequantised weight is never rounded (fp32 accuracy, no per-element FMA).
//
// k-permutation: lane (g = lane/4, c = lane%4) reads words 2c, 2c+1 of a group, i.e.
// elements 16c..16c+15. MMA j (j = 0..3) of a group uses the nibble pairs
// (j, j+4) of both words, so its k-slots 2c, 2c+1, 2c+8, 2c+9 hold elements
// 16c+j, 16c+j+4, 16c+8+j, 16c+12+j. The activation tile is stored in shared memory
// already permuted this way, so B fragments are two 16-byte loads per lane per group.
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

template <bool GATED>
struct Tile {
  static constexpr int kMTiles = 4;              // m16 tiles per warp
  static constexpr int kRows = GATED ? 32 : 64;  // weight rows per matrix per CTA
  static constexpr int kMats = GATED ? 2 : 1;
  static constexpr int kScRows = kRows * kMats;  // rows with scale entries
};

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

// Shared memory: [xs: TOK rows x (2K + 16) bytes][xsum: TOK x G floats], padded to at
// least the cross-warp reduction buffer (which reuses it after the K loop), then
// [sc: kScRows x G float2] at a.sc_offset (kept across token chunks).
//
// Memory-level parallelism: each warp owns a contiguous run of K groups and keeps a ring
// of kPF groups of weight loads in flight (kPF x 4 m16 tiles x 2 rows x 8 bytes per
// lane); the loads for the first kPF groups are issued before the shared-memory staging
// of scales and activations, so their latency overlaps it.
template <bool GATED, int NT8>
__global__ void __launch_bounds__(128, 2) qgemv_kernel(QgemvArgs a) {
  using TL = Tile<GATED>;
  constexpr int TOK = 8 * NT8;
  constexpr int kPF = 4;
  constexpr int MT = TL::kMTiles;
  extern __shared__ __align__(16) unsigned char smem[];
  const int K = a.K, N = a.N;
  const int G = K >> 6;
  const int xs_stride = 2 * K + 16;  // bytes per token row (padding breaks bank conflicts)
  unsigned char* xs = smem;
  float* xsum = reinterpret_cast<float*>(smem + (size_t)TOK * xs_stride);
  float2* sc = reinterpret_cast<float2*>(smem + a.sc_offset);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gq = lane >> 2, cq = lane & 3;

  // ---- expert / rows of this CTA
  const int slot = blockIdx.y;
  if (a.n_active && slot >= *a.n_active) return;
  const int e = a.active ? a.active[slot] : slot;
  const int64_t row_begin = a.offsets ? a.offsets[e] : 0;
  const int64_t row_end = a.offsets ? a.offsets[e + 1] : a.n_identity;
  if (row_end <= row_begin) return;
  const int n0 = blockIdx.x * TL::kRows;
  const RowMap rm{a.x_mode, a.x_repeat, a.lhs, a.perm};

  // ---- per-lane weight row pointers (rows gq and gq+8 of each m16 tile)
  const uint32_t* wp_lo[MT];
  const uint32_t* wp_hi[MT];
  bool ok_lo[MT], ok_hi[MT];
  int scr_lo[MT], scr_hi[MT];  // sc row index
  const int wpr = K >> 3;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const int mat = GATED ? (mt >> 1) : 0;
    const int rloc = GATED ? (mt & 1) * 16 : mt * 16;
    const uint32_t* W = mat ? a.w1 : a.w0;
    const int rlo = n0 + rloc + gq, rhi = rlo + 8;
    ok_lo[mt] = rlo < N;
    ok_hi[mt] = rhi < N;
    wp_lo[mt] = W + ((size_t)e * N + (ok_lo[mt] ? rlo : 0)) * wpr + 2 * cq;
    wp_hi[mt] = W + ((size_t)e * N + (ok_hi[mt] ? rhi : 0)) * wpr + 2 * cq;
    scr_lo[mt] = mat * TL::kRows + rloc + gq;
    scr_hi[mt] = scr_lo[mt] + 8;
  }
  const int gpw = (G + kWarps - 1) / kWarps;
  const int g_begin = min(G, warp * gpw);
  const int g_end = min(G, g_begin + gpw);

  uint2 wl[kPF][MT], wh[kPF][MT];
  auto load_group = [&](int slotp, int g) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const bool go = g < g_end;
      wl[slotp][mt] = (go && ok_lo[mt]) ? ldg_nc_u2(wp_lo[mt] + g * 8) : make_uint2(0, 0);
      wh[slotp][mt] = (go && ok_hi[mt]) ? ldg_nc_u2(wp_hi[mt] + g * 8) : make_uint2(0, 0);
    }
  };

  bool first_chunk = true;
  for (int64_t cbase = row_begin; cbase < row_end; cbase += TOK) {
    const int ntok = (row_end - cbase < TOK) ? (int)(row_end - cbase) : TOK;
    // ---- issue the first kPF groups of weight loads
#pragma unroll
    for (int i = 0; i < kPF; ++i) load_group(i, g_begin + i);
    __syncthreads();  // previous chunk's readers of xs / the reduction buffer are done
    if (first_chunk) {
      // ---- scales: sc[r][g] = (s, b - 128 s); 16-byte loads of 8 groups of one row
      const int cpr = (G + 7) >> 3;  // 8-group chunks per row
      for (int idx = tid; idx < TL::kScRows * cpr; idx += 128) {
        const int r = idx / cpr, c8 = idx - r * cpr;
        const int mat = r / TL::kRows;
        const int row = n0 + (r - mat * TL::kRows);
        const uint16_t* S = mat ? a.s1 : a.s0;
        const uint16_t* B = mat ? a.b1 : a.b0;
        const size_t off = ((size_t)e * N + (row < N ? row : 0)) * G + c8 * 8;
        const int ng = min(8, G - c8 * 8);
        uint16_t sv[8], bv[8];
        if (ng == 8 && (off & 7) == 0) {
          const uint4 s4 = *reinterpret_cast<const uint4*>(S + off);
          const uint4 b4 = B ? *reinterpret_cast<const uint4*>(B + off) : make_uint4(0, 0, 0, 0);
          const uint32_t su[4] = {s4.x, s4.y, s4.z, s4.w}, bu[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            sv[2 * i] = (uint16_t)(su[i] & 0xffff); sv[2 * i + 1] = (uint16_t)(su[i] >> 16);
            bv[2 * i] = (uint16_t)(bu[i] & 0xffff); bv[2 * i + 1] = (uint16_t)(bu[i] >> 16);
          }
        } else {
          for (int i = 0; i < 8; ++i) {
            sv[i] = i < ng ? S[off + i] : 0;
            bv[i] = (i < ng && B) ? B[off + i] : 0;
          }
        }
        for (int i = 0; i < ng; ++i) {
          float s = 0.0f, cb = 0.0f;
          if (row < N) {
            s = bf2f(sv[i]);
            cb = __fmaf_rn(-128.0f, s, bf2f(bv[i]));
          }
          sc[r * G + c8 * 8 + i] = make_float2(s, cb);
        }
      }
      first_chunk = false;
    }
    // ---- stage the valid token rows: permuted bf16 tile + per-group sums. Rows past
    // ntok are not written: a column of the MMA result depends on its own token only,
    // and those columns are never stored.
    const int units = ntok * G * 4;
    for (int u0 = 0; u0 < units; u0 += 128) {  // uniform trip count: the shuffles need all lanes
      const int u = u0 + tid;
      const bool uvalid = u < units;
      const int c = u & 3;
      const int g = (u >> 2) % G;
      const int t = (u >> 2) / G;
      uint32_t in[8];
      if (uvalid) {
        const int64_t xr = rm.xrow(cbase + t);
        const uint4* src = reinterpret_cast<const uint4*>(a.x + (size_t)xr * K + g * 64 + c * 16);
        const uint4 v0 = src[0], v1 = src[1];
        in[0] = v0.x; in[1] = v0.y; in[2] = v0.z; in[3] = v0.w;
        in[4] = v1.x; in[5] = v1.y; in[6] = v1.z; in[7] = v1.w;
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) in[i] = 0u;
      }
      float ps = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) ps = __fadd_rn(__fadd_rn(ps, bf_lo(in[i])), bf_hi(in[i]));
      uint4 o0, o1;
      o0.x = __byte_perm(in[0], in[2], 0x5410);  // j=0: (e0, e4)
      o0.y = __byte_perm(in[4], in[6], 0x5410);  //      (e8, e12)
      o0.z = __byte_perm(in[0], in[2], 0x7632);  // j=1: (e1, e5)
      o0.w = __byte_perm(in[4], in[6], 0x7632);  //      (e9, e13)
      o1.x = __byte_perm(in[1], in[3], 0x5410);  // j=2: (e2, e6)
      o1.y = __byte_perm(in[5], in[7], 0x5410);  //      (e10, e14)
      o1.z = __byte_perm(in[1], in[3], 0x7632);  // j=3: (e3, e7)
      o1.w = __byte_perm(in[5], in[7], 0x7632);  //      (e11, e15)
      if (uvalid) {
        uint4* dst = reinterpret_cast<uint4*>(xs + (size_t)t * xs_stride + g * 128 + c * 32);
        dst[0] = o0;
        dst[1] = o1;
      }
      ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, 1));
      ps = __fadd_rn(ps, __shfl_xor_sync(0xffffffffu, ps, 2));
      if (uvalid && c == 0) xsum[t * G + g] = ps;
    }
    __syncthreads();

    // ---- main loop over this warp's groups with a kPF-deep ring of weight loads
    float acc[MT][NT8][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int n = 0; n < NT8; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[mt][n][i] = 0.0f;
    const bool n1_live = NT8 > 1 && ntok > 8;
    for (int gb = g_begin; gb < g_end; gb += kPF) {
#pragma unroll
      for (int i = 0; i < kPF; ++i) {
        const int g = gb + i;
        if (g < g_end) {
          uint32_t bf[NT8][8];
          float X0[NT8], X1[NT8];
#pragma unroll
          for (int n = 0; n < NT8; ++n) {
            if (n == 0 || n1_live) {
              const uint4* src =
                  reinterpret_cast<const uint4*>(xs + (size_t)(n * 8 + gq) * xs_stride + g * 128 + cq * 32);
              const uint4 v0 = src[0], v1 = src[1];
              bf[n][0] = v0.x; bf[n][1] = v0.y; bf[n][2] = v0.z; bf[n][3] = v0.w;
              bf[n][4] = v1.x; bf[n][5] = v1.y; bf[n][6] = v1.z; bf[n][7] = v1.w;
              X0[n] = xsum[(n * 8 + 2 * cq) * G + g];
              X1[n] = xsum[(n * 8 + 2 * cq + 1) * G + g];
            }
          }
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            const float2 slo = sc[scr_lo[mt] * G + g];
            const float2 shi = sc[scr_hi[mt] * G + g];
            float d[NT8][4];
#pragma unroll
            for (int n = 0; n < NT8; ++n)
#pragma unroll
              for (int q = 0; q < 4; ++q) d[n][q] = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t a0 = nib_pair(wl[i][mt].x, j), a1 = nib_pair(wh[i][mt].x, j);
              const uint32_t a2 = nib_pair(wl[i][mt].y, j), a3 = nib_pair(wh[i][mt].y, j);
#pragma unroll
              for (int n = 0; n < NT8; ++n)
                if (n == 0 || n1_live) mma_bf16_16816(d[n], a0, a1, a2, a3, bf[n][2 * j], bf[n][2 * j + 1]);
            }
#pragma unroll
            for (int n = 0; n < NT8; ++n) {
              if (n == 0 || n1_live) {
                acc[mt][n][0] = __fmaf_rn(slo.y, X0[n], __fmaf_rn(slo.x, d[n][0], acc[mt][n][0]));
                acc[mt][n][1] = __fmaf_rn(slo.y, X1[n], __fmaf_rn(slo.x, d[n][1], acc[mt][n][1]));
                acc[mt][n][2] = __fmaf_rn(shi.y, X0[n], __fmaf_rn(shi.x, d[n][2], acc[mt][n][2]));
                acc[mt][n][3] = __fmaf_rn(shi.y, X1[n], __fmaf_rn(shi.x, d[n][3], acc[mt][n][3]));
              }
            }
          }
          load_group(i, g + kPF);
        }
      }
    }

    // ---- cross-warp reduction (warp order 0,1,2,3) through shared memory
    __syncthreads();  // everyone is done reading xs and xsum for this chunk
    float* red = reinterpret_cast<float*>(smem);
    constexpr int kPer = MT * NT8 * 4;
    if (warp > 0) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int n = 0; n < NT8; ++n)
#pragma unroll
          for (int i = 0; i < 4; ++i) red[((warp - 1) * kPer + (mt * NT8 + n) * 4 + i) * 32 + lane] = acc[mt][n][i];
    }
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int w = 0; w < kWarps - 1; ++w)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
          for (int n = 0; n < NT8; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i)
              acc[mt][n][i] = __fadd_rn(acc[mt][n][i], red[(w * kPer + (mt * NT8 + n) * 4 + i) * 32 + lane]);
      // ---- epilogue: C fragment (row gq / gq+8, tokens 2cq / 2cq+1)
#pragma unroll
      for (int n = 0; n < NT8; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int t = n * 8 + 2 * cq + (i & 1);
          if (t < ntok) {
            const int64_t pos = cbase + t;
            const int64_t orow = a.out_mode == 0 ? pos : rm.orig(pos);
            uint16_t* o = a.out + (size_t)orow * N;
            const int rsub = gq + ((i >> 1) << 3);
            if (GATED) {
#pragma unroll
              for (int mt = 0; mt < 2; ++mt) {
                const int row = n0 + mt * 16 + rsub;
                if (row < N) o[row] = swiglu_bf16(rbf(acc[mt][n][i]), rbf(acc[mt + 2][n][i]));
              }
            } else {
#pragma unroll
              for (int mt = 0; mt < MT; ++mt) {
                const int row = n0 + mt * 16 + rsub;
                if (row < N) o[row] = f2bf(acc[mt][n][i]);
              }
            }
          }
        }
    }
  }
}

template <bool GATED, int NT8>
static cudaError_t launch_qgemv_t(const QgemvArgs& a, int slots, cudaStream_t st) {
  using TL = Tile<GATED>;
  constexpr int TOK = 8 * NT8;
  const int G = a.K / 64;
  // Layout: [xs | xsum] padded up to the reduction buffer size, then sc.
  const size_t front = std::max((size_t)TOK * (2 * a.K + 16) + sizeof(float) * TOK * G,
                                sizeof(float) * (kWarps - 1) * TL::kMTiles * NT8 * 4 * 32);
  const size_t smem = front + sizeof(float2) * TL::kScRows * G;
  if (smem > 227 * 1024) return cudaErrorInvalidConfiguration;
  auto kern = qgemv_kernel<GATED, NT8>;
  // Raise the dynamic shared memory limit once per device and size (not per launch).
  static thread_local int set_dev = -1;
  static thread_local size_t set_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != set_dev || smem > set_smem) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    if (err != cudaSuccess) return err;
    set_dev = dev;
    set_smem = 227 * 1024;
  }
  dim3 grid((a.N + TL::kRows - 1) / TL::kRows, slots);
  QgemvArgs b = a;
  b.sc_offset = (int)front;
  kern<<<grid, 128, smem, st>>>(b);
  return cudaGetLastError();
}

cudaError_t launch_qgemv(const QgemvArgs& a, bool gated, int slots, int max_rows_per_expert,
                         cudaStream_t st) {
  if (slots <= 0) return cudaSuccess;
  const bool small = max_rows_per_expert <= 8;
  if (gated) return small ? launch_qgemv_t<true, 1>(a, slots, st) : launch_qgemv_t<true, 2>(a, slots, st);
  return small ? launch_qgemv_t<false, 1>(a, slots, st) : launch_qgemv_t<false, 2>(a, slots, st);
}

}  // namespace moe
