// qgemm_tc.cu — grouped 4-bit GEMM on tcgen05 tensor cores (prefill regime).
//
// Replaces gather_qmm / quantized_matmul (crates/mlx-core/src/ops.rs:592-637, 830-891)
// for the SwitchGLU gate/up/down projections (qwen3_moe_python_port.rs:311-359) and the
// shared expert (:385-390) when experts see many tokens.
//
// One CTA computes D[128 weight rows x n tokens] = W_tile . X_tile^T over the whole K
// for one expert and one tile of up to 256 of its (grouped) token rows:
//   * warps 0-15 (512 threads) are producers: per K step of 64 (one quantization group)
//     thread p loads 16 packed int4 elements of weight row p/4 (quarter p%4 of the group),
//     dequantises them to bf16 (w = RN_bf16(s*q + b), the value MLX's GPU qmm computes
//     into threadgroup memory) and stores them into the A tile, and copies its share of
//     the token rows with cp.async into the B tile; both tiles are K-major with the
//     128-byte swizzle the tensor core reads;
//   * warp 16 allocates tensor memory and, from one lane, issues tcgen05.mma
//     (kind::f16, bf16 x bf16 -> fp32, M=128, N=n rounded up to 16, K=16 per instruction)
//     accumulating in TMEM; tcgen05.commit on an mbarrier frees each stage;
//   * after the last stage the producer warps read the accumulators back with
//     tcgen05.ld (warp w owns TMEM lanes 32(w%4).. = weight rows, and every fourth block
//     of 32 token columns by w/4); in the gated form the gate and up accumulators (TMEM
//     columns 0 and 256) are combined by SwiGLU in registers (bf16 multiplies exact as in
//     the reference; the sigmoid from the hardware ex2/rcp approximations, which is why
//     this path has its own tolerance against the oracle). Each warp transposes its
//     32 x 32 tile through shared memory so that the outputs leave as 16-byte stores.
//   * warp 17 streams the packed weights: per K step, one 2D TMA load
//     (cp.async.bulk.tensor) of the [128 rows][32 bytes] tile of each matrix into a slot
//     of a kPackSlots-deep ring (full: the TMA's bytes landed; empty: every producer
//     warp read its words), so the producers dequantise from shared memory instead of
//     waiting on global loads.
// The shared-memory ring has kStages stages guarded by full/empty mbarriers. Every
// mbarrier wait is bounded; on expiry the CTA records a status code and drains out (the
// TMA warp waits for its copies in flight before the CTA exits). The TMA loads are plain
// loads of this GPU's memory, never with cluster multicast.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "kernels.cuh"

namespace moe {

namespace {

constexpr int kBM = 128;                   // weight rows per CTA (MMA M)
constexpr int kBN = kTcTileRows;           // max tokens per CTA (MMA N)
constexpr int kBK = 64;                    // K per stage
constexpr int kATileBytes = kBM * kBK * 2;   // 16 KB
constexpr int kBTileBytes = kBN * kBK * 2;   // 32 KB
constexpr int kProducers = 512;
constexpr int kParts = kProducers / kBM;    // producer threads per weight row (4)
constexpr int kWords = 8 / kParts;          // packed words of a group each handles (2)
constexpr int kColGroups = kProducers / 128;  // epilogue: warps sharing a TMEM lane quadrant
constexpr int kMmaWarp = kProducers / 32;
constexpr int kTmaWarp = kMmaWarp + 1;        // streams the packed weight tiles
constexpr int kThreads = kProducers + 64;
constexpr int kPackSlots = 4;                 // K steps of packed weights in flight
constexpr int kPackTileBytes = kBM * 32;      // [128 rows][8 words] of one matrix, one K step
constexpr uint64_t kWaitLimitNs = 200ull * 1000 * 1000;  // bound of one mbarrier wait (200 ms)
#ifndef MOE_TC_WAIT_SLEEP_NS
#define MOE_TC_WAIT_SLEEP_NS 2000
#endif
constexpr uint32_t kWaitSleepNs = MOE_TC_WAIT_SLEEP_NS;  // suspend hint of one try_wait in a wait loop

// MODE 0: plain, 128 weight rows per CTA; 1: gated (gate and up rows); 2: plain, 256
// weight rows per CTA as two 128-row accumulators (halves the token-tile reloads).
template <int MODE>
struct TcCfg {
  static constexpr int kMats = MODE ? 2 : 1;
  static constexpr int kStages = MODE ? 3 : 4;
  static constexpr int kStageBytes = kMats * kATileBytes + kBTileBytes;
  static constexpr int kTmemCols = MODE ? 512 : 256;
  // [stages][A tiles..., B tile] | [pack slots][matrices][128 rows][32 B] |
  // full[S] empty[S] done pfull[P] pempty[P] | tmem base | xrow[kBN]
  static constexpr int kPackOffset = kStages * kStageBytes;
  static constexpr int kBarOffset = kPackOffset + kPackSlots * kMats * kPackTileBytes;
  static constexpr int kNumBars = 2 * kStages + 1 + 2 * kPackSlots;
  static constexpr int kSmemBytes = kBarOffset + 8 * kNumBars + 16 + 4 * kBN + 1024;
};

MOE_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

MOE_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count) : "memory");
}
MOE_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
MOE_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait that may suspend the thread in hardware for up to `ns` nanoseconds while the
// phase is incomplete (instead of returning at once), so that waiting warps leave the
// issue slots to the warps with work
MOE_DEV bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
MOE_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}
// Bounded wait: false when the limit expired (the caller records it and drains out).
MOE_DEV bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait_sleep(bar, parity, kWaitSleepNs))
    if (global_ns() - t0 > kWaitLimitNs) return false;
  return true;
}

MOE_DEV void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
// 2D tiled TMA load of the box at (x, y) of the tensor map into shared memory, completing
// on bar. A plain load: no cluster multicast (this kernel also runs under expert
// parallelism).
MOE_DEV void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

MOE_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }
MOE_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
MOE_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

MOE_DEV void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src));
}
MOE_DEV void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
MOE_DEV void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 bytes
// apart (SBO), Blackwell descriptor version 1.
MOE_DEV uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fffu);
  d |= (uint64_t)1 << 16;           // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset
  d |= (uint64_t)1 << 46;           // version
  d |= (uint64_t)2 << 61;           // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: bf16 A and B (K-major), fp32 accumulate, M=128.
MOE_DEV uint32_t idesc_bf16(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

MOE_DEV void tc_mma(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
MOE_DEV void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
               : "memory");
}

MOE_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

MOE_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// bf16 pair (128 + q_j, 128 + q_{j+4}) from nibbles j and j+4 of w.
MOE_DEV uint32_t nib_pair(uint32_t w, int j) {
  uint32_t r;
  const uint32_t v = w >> (4 * j);
  asm("lop3.b32 %0, %1, %2, %3, 0xea;\n" : "=r"(r) : "r"(v), "r"(0x000f000fu), "r"(0x43004300u));
  return r;
}

MOE_DEV uint32_t bf2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
MOE_DEV uint32_t bf2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;\n" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

// Eight 4-bit fields of w (element order 0..7) -> eight bf16 values RN(s*q + b), in
// element order, as four bf16 pairs. s2 / b2 hold (s, s) / (b, b).
MOE_DEV uint4 dequant8(uint32_t w, uint32_t s2, uint32_t b2) {
  const uint32_t t0 = nib_pair(w, 0), t1 = nib_pair(w, 1), t2 = nib_pair(w, 2), t3 = nib_pair(w, 3);
  const uint32_t k128 = 0x43004300u;  // (128, 128)
  uint4 o;
  o.x = bf2_fma(bf2_sub(__byte_perm(t0, t1, 0x5410), k128), s2, b2);  // (e0, e1)
  o.y = bf2_fma(bf2_sub(__byte_perm(t2, t3, 0x5410), k128), s2, b2);  // (e2, e3)
  o.z = bf2_fma(bf2_sub(__byte_perm(t0, t1, 0x7632), k128), s2, b2);  // (e4, e5)
  o.w = bf2_fma(bf2_sub(__byte_perm(t2, t3, 0x7632), k128), s2, b2);  // (e6, e7)
  return o;
}

MOE_DEV uint4 lds_v4(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}

// Two fp32 values -> packed bf16 pair (lo = a), round to nearest even (cvt.rn.bf16x2).
MOE_DEV uint32_t pack_bf2(float a, float b) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;\n" : "=r"(r) : "f"(b), "f"(a));
  return r;
}
MOE_DEV uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;\n" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// sigmoid(x) from the hardware base-2 exponential and reciprocal approximations
// (relative error a few fp32 ulps; the result is rounded to bf16 by the caller).
MOE_DEV float sigmoid_fast(float x) {
  float e, r;
  asm("ex2.approx.ftz.f32 %0, %1;\n" : "=f"(e) : "f"(x * -1.4426950408889634f));
  asm("rcp.approx.ftz.f32 %0, %1;\n" : "=f"(r) : "f"(1.0f + e));
  return r;
}
// SwiGLU of two (gate, up) pairs on the tensor-core path: h = bf16(bf16(g * bf16(sig(g))) * u)
// with g and u first rounded to bf16 (the bf16 outputs of the two projections). The
// products of bf16 values are exact in fp32, so mul.rn.bf16x2 rounds them as the
// reference's bf16 multiplies do; only sigmoid is approximate (see sigmoid_fast).
MOE_DEV uint32_t swiglu2_fast(float g0, float g1, float u0, float u1) {
  const uint32_t g2 = pack_bf2(g0, g1), u2 = pack_bf2(u0, u1);
  const float gr0 = bf_lo(g2), gr1 = bf_hi(g2);
  const uint32_t s2 = pack_bf2(sigmoid_fast(gr0), sigmoid_fast(gr1));
  return bf2_mul(bf2_mul(g2, s2), u2);
}

// Byte offset of 16-byte chunk c of row r in a 128-byte-swizzled K-major tile.
MOE_DEV uint32_t sw128_off(int r, int c) { return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4)); }

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

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) tc_gemm_kernel(const __grid_constant__ TcGemmArgs ta) {
  using C = TcCfg<MODE>;
  constexpr bool GATED = MODE == 1;
  constexpr int kRowsPerCta = MODE == 2 ? 2 * kBM : kBM;
  const QgemvArgs& a = ta.q;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar_full = sbase + C::kBarOffset;
  const uint32_t bar_empty = bar_full + 8 * C::kStages;
  const uint32_t bar_done = bar_empty + 8 * C::kStages;
  const uint32_t bar_pfull = bar_done + 8;                  // packed slot landed (TMA bytes)
  const uint32_t bar_pempty = bar_pfull + 8 * kPackSlots;   // packed slot read by every producer warp
  const uint32_t pack_s = sbase + C::kPackOffset;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kBarOffset + 8 * C::kNumBars);
  int32_t* xrow_s = reinterpret_cast<int32_t*>(smem + C::kBarOffset + 8 * C::kNumBars + 16);
  __shared__ int abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int K = a.K, N = a.N, Gtot = K >> 6;
  // split-K (blockIdx.z): this CTA accumulates K steps [G0, G0 + G) of the Gtot
  const int ksp = ta.ksplit > 1 ? ta.ksplit : 1;
  const int spk = (Gtot + ksp - 1) / ksp;
  const int G0 = (int)blockIdx.z * spk;
  const int G = (G0 + spk < Gtot ? G0 + spk : Gtot) - G0;
  const int n0 = blockIdx.x * kRowsPerCta;

  pdl_wait();
  // ---- map blockIdx.y to (expert, token tile)
  const int w = blockIdx.y;
  int e = 0;
  int64_t tbeg, tend;
  if (ta.tile_start) {
    // tile_start has E + 1 entries: find e with tile_start[e] <= w < tile_start[e + 1]
    int l = 0, r = ta.num_experts;
    if (w >= ta.tile_start[r]) return;
    while (r - l > 1) {
      const int m = (l + r) >> 1;
      if (ta.tile_start[m] <= w) l = m;
      else r = m;
    }
    e = l;
    tbeg = a.offsets[e] + (int64_t)(w - ta.tile_start[e]) * kBN;
    const int64_t eend = a.offsets[e + 1];
    tend = (tbeg + kBN < eend) ? tbeg + kBN : eend;
  } else {
    tbeg = (int64_t)w * kBN;
    if (tbeg >= a.n_identity) return;
    tend = (tbeg + kBN < a.n_identity) ? tbeg + kBN : a.n_identity;
  }
  const int ntok = (int)(tend - tbeg);
  const int nmma = (ntok + 15) & ~15;
  const RowMap rm{a.x_mode, a.x_repeat, a.lhs, a.perm};

  // ---- setup: barriers, token row indices, TMEM
  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(bar_full + 8 * s, kProducers);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_done, 1);
    for (int i = 0; i < kPackSlots; ++i) {
      mbar_init(bar_pfull + 8 * i, 1);
      mbar_init(bar_pempty + 8 * i, kMmaWarp);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  for (int i = tid; i < kBN; i += kThreads) xrow_s[i] = i < ntok ? (int32_t)rm.xrow(tbeg + i) : -1;
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(C::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < kMmaWarp) {
    // ================= producers (then epilogue) =================
    const int p = tid;               // 0..kProducers-1
    const int part = p % kParts;     // which kWords words (8 elements each) of the row's group
    const int row = p / kParts;      // weight row within the tile
    const uint16_t* srow[C::kMats];
    const uint16_t* brow[C::kMats];
#pragma unroll
    for (int m = 0; m < C::kMats; ++m) {
      const size_t grow = (size_t)e * N + n0 + (MODE == 2 ? m * kBM : 0) + row;
      const bool second = GATED && m;
      const uint16_t* S = second ? a.s1 : a.s0;
      const uint16_t* B = second ? a.b1 : a.b0;
      srow[m] = S + grow * Gtot + G0;
      brow[m] = B ? B + grow * Gtot + G0 : nullptr;
    }
    // register ring of (scale | bias << 16), kRing - 1 stages ahead; the packed weights
    // come from the slots the TMA warp fills (this thread: 8 bytes of row `row`)
    static_assert(kWords == 2, "the slot reads below move 2 words per matrix");
    constexpr int kRing = 4;
    uint32_t sr[kRing][C::kMats];
    auto load_w = [&](int slot3, int kk) {
      if (kk < G) {
#pragma unroll
        for (int m = 0; m < C::kMats; ++m) {
          const uint32_t sv = __ldg(srow[m] + kk);
          const uint32_t bv = brow[m] ? __ldg(brow[m] + kk) : 0u;
          sr[slot3][m] = sv | (bv << 16);
        }
      }
    };
    // B tile: 256 rows x 8 chunks of 16 bytes; this thread copies chunks q = p + kProducers i
    // (rows fixed for the whole K loop, so their source rows and tile offsets are formed once)
    constexpr int kBChunks = kBN * 8 / kProducers;
    const uint16_t* bsrc[kBChunks];
    uint32_t bdst[kBChunks];
#pragma unroll
    for (int i = 0; i < kBChunks; ++i) {
      const int q = p + kProducers * i;
      const int r = q >> 3, c = q & 7;
      bdst[i] = sw128_off(r, c);
      bsrc[i] = r < ntok ? a.x + (size_t)xrow_s[r] * K + (size_t)G0 * kBK + c * 8 : nullptr;
    }
    auto issue_b = [&](int kk) {
      const uint32_t bt = sbase + (kk % C::kStages) * C::kStageBytes + C::kMats * kATileBytes;
#pragma unroll
      for (int i = 0; i < kBChunks; ++i)
        if (bsrc[i]) cp_async16(bt + bdst[i], bsrc[i] + kk * kBK);
      cp_commit();
    };
    constexpr int LA = C::kStages - 1;  // B tiles issued this many stages ahead
    bool ok = true;
#pragma unroll
    for (int i = 0; i < kRing - 1; ++i) load_w(i, i);
    for (int kk = 0; kk < LA; ++kk) {
      if (kk < G) {
        // fresh barriers: the first wait on "empty" passes immediately
        issue_b(kk);
      } else {
        cp_commit();
      }
    }
    for (int kb = 0; kb < G && ok; kb += kRing) {
#pragma unroll
      for (int r3 = 0; r3 < kRing; ++r3) {
        const int kk = kb + r3;
        if (kk < G && ok) {
          const int s = kk % C::kStages;
          const uint32_t st = sbase + s * C::kStageBytes;
          // the packed weights of K step kk: slot kk % kPackSlots, then release the slot
          const int ps = kk % kPackSlots;
          if (!__all_sync(0xffffffffu, mbar_wait(bar_pfull + 8 * ps, (kk / kPackSlots) & 1))) {
            ok = false;  // warp-uniform: the whole warp leaves together
            if (lane == 0) atomicOr(&abort_flag, 16);
            break;
          }
          uint2 wr[C::kMats];
#pragma unroll
          for (int m = 0; m < C::kMats; ++m) {
            const uint32_t src = pack_s + (uint32_t)((ps * C::kMats + m) * kPackTileBytes + row * 32 + part * 8);
            asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];\n" : "=r"(wr[m].x), "=r"(wr[m].y) : "r"(src) : "memory");
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_pempty + 8 * ps);
          // dequantise A(kk) into stage s (freed: its empty barrier was awaited when B(kk) was issued)
#pragma unroll
          for (int m = 0; m < C::kMats; ++m) {
            const uint32_t sv = sr[r3][m] & 0xffffu, bv = sr[r3][m] >> 16;
            const uint32_t s2 = sv | (sv << 16), b2 = bv | (bv << 16);
            const uint2 wv = wr[m];
            const uint32_t ws[2] = {wv.x, wv.y};
#pragma unroll
            for (int j = 0; j < kWords; ++j) {
              const uint4 o = dequant8(ws[j], s2, b2);
              const uint32_t dst = st + m * kATileBytes + sw128_off(row, part * kWords + j);
              asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};\n" ::"r"(dst), "r"(o.x), "r"(o.y), "r"(o.z),
                           "r"(o.w)
                           : "memory");
            }
          }
          load_w((r3 + kRing - 1) % kRing, kk + kRing - 1);
          // B(kk) landed: at most LA-1 newer groups may still be pending
          cp_wait<LA - 1>();
          fence_proxy_async();
          mbar_arrive(bar_full + 8 * s);
          // issue B(kk + LA) into the stage MMA(kk + LA - kStages) releases
          const int kn = kk + LA;
          if (kn < G) {
            const int sn = kn % C::kStages;
            const int use = kn / C::kStages;  // this is use number `use` of stage sn
            if (use > 0 && !__all_sync(0xffffffffu, mbar_wait(bar_empty + 8 * sn, (use - 1) & 1))) {
              ok = false;  // warp-uniform (the slot reads above synchronise the warp)
              if (lane == 0) atomicOr(&abort_flag, 1);
            }
            if (ok) issue_b(kn);
          } else {
            cp_commit();
          }
        }
      }
    }
    cp_wait<0>();
    // ================= epilogue =================
    const bool done_ok = __all_sync(0xffffffffu, ok && mbar_wait(bar_done, 0));  // warp-uniform for tcgen05.ld
    if (!done_ok && lane == 0) atomicOr(&abort_flag, 2);
    tc_fence_after();
    pdl_trigger();
    if (done_ok && ksp > 1) {
      // split-K: fp32 partials [kz][pos][N] (plain) or [kz][pos][gate N | up N] (gated),
      // added in split order and finished by the GEMV's reduction kernel
      const int quad = warp & 3;
      const uint32_t tl = tmem + ((uint32_t)(32 * quad) << 16);
      const int N2 = GATED ? 2 * N : N;
      for (int c0 = 32 * (warp >> 2); c0 < nmma; c0 += 32 * kColGroups) {
#pragma unroll 1
        for (int m = 0; m < C::kMats; ++m) {
          const int col = (GATED ? m * N : (MODE == 2 ? m * kBM : 0)) + n0 + 32 * quad + lane;
          float* base = a.partial + ((size_t)blockIdx.z * a.part_rows + (size_t)tbeg) * N2 + col;
#pragma unroll 1
          for (int h = 0; h < 32; h += 16) {
            uint32_t g[16];
            tmem_ld16(tl + m * 256 + c0 + h, g);
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (c0 + h + j < ntok) base[(size_t)(c0 + h + j) * N2] = __uint_as_float(g[j]);
          }
        }
      }
    } else if (done_ok) {
      // Every MMA has completed, so the stage buffers are free: each warp transposes its
      // 32 rows x 32 tokens tile through 2 KB of stage 0.
      const int quad = warp & 3;                    // TMEM lanes 32*quad.. (weight rows)
      const uint32_t tl = tmem + ((uint32_t)(32 * quad) << 16);
      unsigned char* tile = smem + warp * 2048;     // [32 tokens][32 rows] bf16
      const uint32_t tile_s = sbase + warp * 2048;
      // token row t of the tile = 64 bytes = 4 x 16 bytes; lane -> (t = lane/4 + 8i, piece
      // lane%4); col_off selects the 128-row accumulator (MODE 2)
      int c0 = 0;
      auto store_tile = [&](int col_off) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int t = (lane >> 2) + 8 * i;
          const int tok = c0 + t;
          if (tok < ntok) {
            const uint4 v = lds_v4(tile_s + t * 64 + (lane & 3) * 16);
            const int64_t pos = tbeg + tok;
            const int64_t orow = a.out_mode == 0 ? pos : rm.orig(pos);
            *reinterpret_cast<uint4*>(a.out + (size_t)orow * N + n0 + col_off + 32 * quad + (lane & 3) * 8) = v;
          }
        }
        __syncwarp();
      };
      for (c0 = 32 * (warp >> 2); c0 < nmma; c0 += 32 * kColGroups) {
        uint32_t g[32];
        tmem_ld32(tl + c0, g);
        if (GATED) {
          uint32_t u[32];
          tmem_ld32(tl + 256 + c0, u);
          if (a.act) {  // GELU-tanh(gate) * up in f32 (the Gemma4 SwitchGLU)
#pragma unroll
            for (int j = 0; j < 32; ++j)
              *reinterpret_cast<uint16_t*>(tile + j * 64 + lane * 2) =
                  gelu_mul_bf16(rbf(__uint_as_float(g[j])), rbf(__uint_as_float(u[j])));
          } else {
#pragma unroll
            for (int j = 0; j < 32; j += 2) {
              const uint32_t h2 = swiglu2_fast(__uint_as_float(g[j]), __uint_as_float(g[j + 1]),
                                               __uint_as_float(u[j]), __uint_as_float(u[j + 1]));
              *reinterpret_cast<uint16_t*>(tile + j * 64 + lane * 2) = (uint16_t)(h2 & 0xffffu);
              *reinterpret_cast<uint16_t*>(tile + (j + 1) * 64 + lane * 2) = (uint16_t)(h2 >> 16);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const uint32_t o2 = pack_bf2(__uint_as_float(g[j]), __uint_as_float(g[j + 1]));
            *reinterpret_cast<uint16_t*>(tile + j * 64 + lane * 2) = (uint16_t)(o2 & 0xffffu);
            *reinterpret_cast<uint16_t*>(tile + (j + 1) * 64 + lane * 2) = (uint16_t)(o2 >> 16);
          }
        }
        __syncwarp();
        store_tile(0);
        if (MODE == 2) {  // the second 128-row accumulator
          tmem_ld32(tl + 256 + c0, g);
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const uint32_t o2 = pack_bf2(__uint_as_float(g[j]), __uint_as_float(g[j + 1]));
            *reinterpret_cast<uint16_t*>(tile + j * 64 + lane * 2) = (uint16_t)(o2 & 0xffffu);
            *reinterpret_cast<uint16_t*>(tile + (j + 1) * 64 + lane * 2) = (uint16_t)(o2 >> 16);
          }
          __syncwarp();
          store_tile(kBM);
        }
      }
    }
  } else if (warp == kTmaWarp) {
    // ================= packed weights by TMA (one lane) =================
    // K step kk: the [128 rows][8 words] tile of each matrix at (x = (G0 + kk) * 8 words,
    // y = e * N + n0 (+ 128 for the second accumulator of mode 2)) into slot kk % kPackSlots,
    // once every producer warp has released the slot's previous use
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      for (int kk = 0; kk < G && ok; ++kk) {
        const int ps = kk % kPackSlots;
        if (kk >= kPackSlots && !mbar_wait(bar_pempty + 8 * ps, ((kk / kPackSlots) - 1) & 1)) {
          ok = false;
          atomicOr(&abort_flag, 32);
          break;
        }
        mbar_expect_tx(bar_pfull + 8 * ps, C::kMats * kPackTileBytes);
#pragma unroll
        for (int m = 0; m < C::kMats; ++m) {
          const int y = e * N + n0 + (MODE == 2 ? m * kBM : 0);
          tma_load_2d(pack_s + (uint32_t)((ps * C::kMats + m) * kPackTileBytes), &ta.wmap[GATED ? m : 0],
                      (G0 + kk) * 8, y, bar_pfull + 8 * ps);
        }
        issued = kk + 1;
      }
      // no copy may still be landing when the CTA exits (producers that gave up early
      // left slots unconsumed): wait for the last copy issued into each slot
      for (int kk = issued - kPackSlots < 0 ? 0 : issued - kPackSlots; kk < issued; ++kk)
        if (!mbar_wait(bar_pfull + 8 * (kk % kPackSlots), (kk / kPackSlots) & 1)) atomicOr(&abort_flag, 32);
    }
  } else if (lane == 0) {
    // ================= MMA issuer (warp 16, one lane) =================
    const uint32_t idesc = idesc_bf16(nmma);
    bool ok = true;
    for (int kk = 0; kk < G; ++kk) {
      const int s = kk % C::kStages;
      if (!mbar_wait(bar_full + 8 * s, (kk / C::kStages) & 1)) {
        ok = false;
        atomicOr(&abort_flag, 4);
        break;
      }
      tc_fence_after();
      const uint32_t st = sbase + s * C::kStageBytes;
      const uint64_t bdesc = sw128_desc(st + C::kMats * kATileBytes);
#pragma unroll
      for (int k16 = 0; k16 < kBK / 16; ++k16) {
        const uint32_t acc = (kk > 0 || k16 > 0) ? 1u : 0u;
        const uint64_t koff = (uint64_t)((k16 * 32) >> 4);  // +32 bytes along K
#pragma unroll
        for (int m = 0; m < C::kMats; ++m) {
          const uint64_t adesc = sw128_desc(st + m * kATileBytes);
          tc_mma(tmem + m * 256, adesc + koff, bdesc + koff, idesc, acc);
        }
      }
      tc_commit(bar_empty + 8 * s);
    }
    tc_commit(bar_done);
    (void)ok;
  }
  tc_fence_before();
  __syncthreads();
  if (abort_flag && tid == 0 && ta.status) atomicOr(ta.status, abort_flag);
  if (warp == kMmaWarp) {
    // Every MMA this CTA issued has completed before its tensor memory is freed: the
    // issuer commits bar_done after its last MMA on every path, including after a
    // producer or the issuer gave up waiting (the epilogue then skipped its own wait).
    if (lane == 0 && !mbar_wait(bar_done, 0) && ta.status) atomicOr(ta.status, 8);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(C::kTmemCols) : "memory");
  }
}

// cuTensorMapEncodeTiled from the driver, looked up once through the runtime (no link
// against libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// The packed weights [rows][K / 8] uint32 as a 2D tensor map with [128 rows][8 words]
// boxes (one K step of one 128-row tile; 32-byte inner extent, 16-byte aligned rows).
static cudaError_t encode_weight_map(CUtensorMap* map, const uint32_t* w, int64_t rows, int K) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  if (reinterpret_cast<uintptr_t>(w) & 15) return cudaErrorInvalidValue;
  const cuuint64_t dims[2] = {(cuuint64_t)(K / 8), (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)(K / 8) * 4};
  const cuuint32_t box[2] = {8, (cuuint32_t)kBM};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(w), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int MODE>
static cudaError_t launch_tc_t(const TcGemmArgs& a, cudaStream_t st) {
  using C = TcCfg<MODE>;
  static thread_local int set_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != set_dev) {
    cudaError_t err = cudaFuncSetAttribute(tc_gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           C::kSmemBytes);
    if (err != cudaSuccess) return err;
    set_dev = dev;
  }
  dim3 grid(a.q.N / (MODE == 2 ? 2 * kBM : kBM), a.max_tiles, a.ksplit > 1 ? a.ksplit : 1);
  return launch_k(tc_gemm_kernel<MODE>, grid, dim3(kThreads), (size_t)C::kSmemBytes, st, a);
}

cudaError_t launch_tc_gemm(const TcGemmArgs& a0, bool gated, cudaStream_t st) {
  if (a0.max_tiles <= 0) return cudaSuccess;
  if (a0.q.N % kBM != 0 || a0.q.K % kBK != 0) return cudaErrorInvalidValue;
  TcGemmArgs a = a0;
  const int64_t rows = (int64_t)(a.tile_start ? a.num_experts : 1) * a.q.N;
  cudaError_t err = encode_weight_map(&a.wmap[0], a.q.w0, rows, a.q.K);
  if (err != cudaSuccess) return err;
  if (gated) {
    err = encode_weight_map(&a.wmap[1], a.q.w1, rows, a.q.K);
    if (err != cudaSuccess) return err;
  } else {
    a.wmap[1] = a.wmap[0];
  }
  err = gated ? launch_tc_t<1>(a, st) : (a.q.N % (2 * kBM) == 0 ? launch_tc_t<2>(a, st) : launch_tc_t<0>(a, st));
  if (err != cudaSuccess || a.ksplit <= 1) return err;
  QgemvArgs r = a.q;
  r.ksplit = a.ksplit;
  return launch_gemv_reduce(r, gated, st);
}

}  // namespace moe
