// router.cu — R1..R4 of the MoE block: router logits, scoring, top-k, combine weights.
//
// Router logits must be bit-identical to the CPU oracle (the expert index sets are
// compared bit for bit), so the router GEMV runs on CUDA cores in the canonical fp32
// order: lane l of a warp owns the 32-element chunks c = l, l+32, ... of K and
// accumulates acc = fma(x[e], w[e], acc) over each chunk in element order, with
// w[e] = fma(scale, q, bias); the 32 lane sums are combined by the xor butterfly
// (offsets 16, 8, 4, 2, 1) and lane 0 holds the result. One warp evaluates NE rows
// against NT tokens at once (independent accumulators, same order for each).
//
// Reference: Linear::forward -> quantized_matmul (crates/mlx-nn/src/linear.rs:117-128),
// softmax (qwen3_moe_python_port.rs:437), argpartition + slice + take_along_axis
// (:438-441), norm_topk_prob (:442-445); LFM2 expert_bias + softmax
// (lfm2_moe_python_port.rs:559-586, 680-686).
#include "common.cuh"
#include "kernels.cuh"
#include "route.cuh"

namespace moe {

template <int NE, int NT>
__global__ void __launch_bounds__(128, 4) router_logits_kernel(RouterArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_wait();
  pdl_trigger();
  router_tile<NE, NT>(a, (blockIdx.x * 4 + warp) * NE, blockIdx.y * NT, lane);
}

// Router logits for large batches. A CTA owns 8 tokens and a range of groups of 4 rows
// (all rows, or a share of them when the tokens alone would not fill the GPU); its warps
// take the groups in turn (group w, w + warps, ...). The CTA first converts its
// 8 token rows once into shared memory as f32 token pairs: row tp (tokens 2tp, 2tp+1)
// holds, per element k, the pair (x[2tp][k], x[2tp+1][k]), so that one 16-byte piece is
// the pairs of elements k and k+1 and a packed fp32x2 fma takes a pair as it is. Piece q
// of a row is stored at q ^ ((q >> 4) & 7), so that the 8 lanes of a quarter warp, which
// read the same piece of consecutive 32-element chunks (16 pieces apart), hit distinct
// banks. Each lane loads a whole 32-element chunk of its rows' packed weights as one
// 16-byte load; dequantised weights w = fma(scale, q, bias) are duplicated into both
// halves of a 64-bit operand, and the 4 x 8 accumulators are 16 packed pairs. The 32
// per-lane sums of a row group are reduced by a transposed butterfly: at offset o each
// lane keeps half of its values, receives the partner's copies of them and adds; that is
// the xor butterfly's tree for every value (fp32 addition commutes), so the logits stay
// bit-identical to router_tile's canonical order, and lane l ends holding value l (row
// l / 8, token l % 8). Two CTAs per SM, so that one CTA's conversion of its token rows
// overlaps the other's arithmetic.
constexpr int kRsTok = 8, kRsRowsPerWarp = 4, kRsMaxWarps = 8;

MOE_DEV void fma2_b64(unsigned long long& acc, unsigned long long x, unsigned long long w) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(x), "l"(w));
}
MOE_DEV unsigned long long dup_f32(float w) {
  unsigned long long r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "f"(w));
  return r;
}
MOE_DEV void lds_v2u64(uint32_t addr, unsigned long long& a, unsigned long long& b) {
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr));
}

// KMAX: the largest K the shared-memory rows hold (row stride KMAX * 8 bytes).
template <int KMAX>
__global__ void __launch_bounds__(kRsMaxWarps * 32, 2) router_logits_smem_kernel(RouterArgs a) {
  extern __shared__ __align__(16) unsigned char xs[];  // [kRsTok / 2][KMAX] (f32, f32)
  constexpr uint32_t kRowBytes = (uint32_t)KMAX * 8;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int K = a.K, nkb = K / 8;
  const int t0 = blockIdx.x * kRsTok;
  const int nt = a.T - t0 < kRsTok ? a.T - t0 : kRsTok;
  pdl_wait();
  for (int i = threadIdx.x; i < (kRsTok / 2) * nkb; i += blockDim.x) {
    const int tp = i / nkb, kb = i - tp * nkb;
    uint4 va = make_uint4(0, 0, 0, 0), vb = make_uint4(0, 0, 0, 0);
    if (2 * tp < nt) va = __ldg(reinterpret_cast<const uint4*>(a.x + (size_t)(t0 + 2 * tp) * K) + kb);
    if (2 * tp + 1 < nt) vb = __ldg(reinterpret_cast<const uint4*>(a.x + (size_t)(t0 + 2 * tp + 1) * K) + kb);
    const uint32_t wa[4] = {va.x, va.y, va.z, va.w}, wb[4] = {vb.x, vb.y, vb.z, vb.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int q = 4 * kb + j;
      *reinterpret_cast<float4*>(xs + tp * kRowBytes + ((q ^ ((q >> 4) & 7)) << 4)) =
          make_float4(bf_lo(wa[j]), bf_lo(wb[j]), bf_hi(wa[j]), bf_hi(wb[j]));
    }
  }
  __syncthreads();
  pdl_trigger();
  const uint32_t xbase = (uint32_t)__cvta_generic_to_shared(xs);
  const int wpr = K >> 3, gpr = K / a.group_size, nchunks = K >> 5;
  // this CTA's row groups: [blockIdx.y * gpc, (blockIdx.y + 1) * gpc)
  const int ngroups = (a.n_rows + kRsRowsPerWarp - 1) / kRsRowsPerWarp;
  const int gpc = (ngroups + gridDim.y - 1) / gridDim.y;
  const int g_end = (blockIdx.y + 1) * gpc < ngroups ? (blockIdx.y + 1) * gpc : ngroups;
  for (int rg = blockIdx.y * gpc + warp; rg < g_end; rg += nwarps) {
    const int row0 = rg * kRsRowsPerWarp;
    unsigned long long acc[kRsRowsPerWarp][kRsTok / 2];  // (token 2tp, token 2tp+1) per row
#pragma unroll
    for (int e = 0; e < kRsRowsPerWarp; ++e)
#pragma unroll
      for (int tp = 0; tp < kRsTok / 2; ++tp) acc[e][tp] = 0ull;
    for (int c = lane; c < nchunks; c += 32) {
      const int g = (c * 32) / a.group_size;
      uint4 wv[kRsRowsPerWarp];
      float sc[kRsRowsPerWarp], bi[kRsRowsPerWarp];
#pragma unroll
      for (int e = 0; e < kRsRowsPerWarp; ++e) {
        // row pointers formed here rather than held across the loop (register pressure)
        const int r = row0 + e;
        const bool is_gate = r >= a.E;  // the extra row is shared_expert_gate
        const int rr = is_gate ? 0 : r;
        const uint16_t* bb = is_gate ? a.gate_b : a.b;
        const bool ok = r < a.n_rows;
        wv[e] = ok ? __ldg(reinterpret_cast<const uint4*>((is_gate ? a.gate_w : a.w) + (size_t)rr * wpr) + c)
                   : make_uint4(0, 0, 0, 0);
        sc[e] = ok ? bf2f(__ldg((is_gate ? a.gate_s : a.s) + (size_t)rr * gpr + g)) : 0.0f;
        bi[e] = (ok && bb) ? bf2f(__ldg(bb + (size_t)rr * gpr + g)) : 0.0f;
      }
      const uint32_t cbase = xbase + (uint32_t)c * 256u;
      const int swz = c & 7;
#pragma unroll 1
      for (int word = 0; word < 4; ++word) {
        uint32_t wd[kRsRowsPerWarp];
#pragma unroll
        for (int e = 0; e < kRsRowsPerWarp; ++e)
          wd[e] = word == 0 ? wv[e].x : word == 1 ? wv[e].y : word == 2 ? wv[e].z : wv[e].w;
        // two element pairs at a time (unrolled further, the loads of later pairs hoisted
        // ahead would take the registers of a second CTA per SM)
#pragma unroll 2
        for (int j = 0; j < 4; ++j) {
          // elements 8 word + 2j and 8 word + 2j + 1 of the chunk, all token pairs
          const uint32_t off = cbase + (uint32_t)(((4 * word + j) ^ swz) << 4);
          unsigned long long xx[kRsTok / 2][2];
#pragma unroll
          for (int tp = 0; tp < kRsTok / 2; ++tp) lds_v2u64(off + tp * kRowBytes, xx[tp][0], xx[tp][1]);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int el = 2 * j + h;
#pragma unroll
            for (int e = 0; e < kRsRowsPerWarp; ++e) {
              // q as an exact float: the field in the mantissa of 2^23, minus 2^23
              const float q = __fsub_rn(__uint_as_float(((wd[e] >> (4 * el)) & 0xfu) | 0x4b000000u), 8388608.0f);
              const unsigned long long ww = dup_f32(__fmaf_rn(sc[e], q, bi[e]));
#pragma unroll
              for (int tp = 0; tp < kRsTok / 2; ++tp) fma2_b64(acc[e][tp], xx[tp][h], ww);
            }
          }
        }
      }
    }
    // transposed butterfly over the 32 values v[e * 8 + t]
    float v[32];
#pragma unroll
    for (int e = 0; e < kRsRowsPerWarp; ++e)
#pragma unroll
      for (int tp = 0; tp < kRsTok / 2; ++tp)
        asm("mov.b64 {%0, %1}, %2;" : "=f"(v[e * 8 + 2 * tp]), "=f"(v[e * 8 + 2 * tp + 1]) : "l"(acc[e][tp]));
#pragma unroll
    for (int lvl = 0; lvl < 5; ++lvl) {
      const int o = 16 >> lvl, n = 32 >> lvl;
      const bool upper = (lane & o) != 0;
#pragma unroll
      for (int j = 0; j < n / 2; ++j) {
        const float send = upper ? v[j] : v[j + n / 2];
        const float keep = upper ? v[j + n / 2] : v[j];
        v[j] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, o));
      }
    }
    const int e = lane >> 3, t = lane & 7;
    if (row0 + e < a.n_rows && t < nt) a.logits[(size_t)(t0 + t) * a.n_rows + row0 + e] = f2bf(v[0]);
  }
}

template <int NE, int NT>
__global__ void __launch_bounds__(128, 4) router_logits_f32_kernel(RouterArgs a) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  pdl_wait();
  pdl_trigger();
  router_tile_f32<NE, NT>(a, (blockIdx.x * 4 + warp) * NE, blockIdx.y * NT, lane);
}

template <int PL>
__global__ void __launch_bounds__(128) topk_kernel(TopkArgs a) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 4 + (threadIdx.x >> 5);
  pdl_wait();
  pdl_trigger();
  if (t >= a.T) return;
  topk_token<PL>(a, t, lane);
}

// ---------------------------------------------------------------------------------
// Fused routing for decode-sized batches: router logits, scoring / top-k and the
// grouping by expert in ONE launch. Every CTA computes its tile of logits; the last CTA
// to finish a token tile (a per-tile ticket counter) runs the top-k of those tokens;
// the last token tile to finish (a global ticket) groups all pairs. No CTA waits for
// another: the work moves to whichever CTA arrives last, after a __threadfence() that
// publishes the arriving CTA's writes. Each last CTA puts its counter back to zero, so
// the counters (in the context's zero-initialised status block) are zero between calls.
// ---------------------------------------------------------------------------------

// Exclusive scan of one value per thread over a 128-thread CTA (thread order).
MOE_DEV int32_t scan128(int32_t v, int32_t* sh, int32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int32_t u = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += u;
  }
  if (lane == 31) sh[warp] = incl;
  __syncthreads();
  int32_t wbase = 0, tot = 0;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    const int32_t x = sh[w];
    if (w < warp) wbase += x;
    tot += x;
  }
  __syncthreads();
  if (total) *total = tot;
  return incl - v + wbase;
}

// Stable grouping of a.P pairs by expert with 128 threads (the semantics of
// launch_group: offsets, active list, n_active, perm, inv, tile_start). wcnt: 4 * E ints.
MOE_DEV void group_cta128(const GroupArgs& a, int32_t* wcnt, int32_t* sh) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int E = a.E;
  for (int i = tid; i < 4 * E; i += 128) wcnt[i] = 0;
  __syncthreads();
  const int64_t seg = (a.P + 3) / 4;
  const int64_t p0 = warp * seg;
  const int64_t p1 = (p0 + seg < a.P) ? p0 + seg : a.P;
  auto key = [&](int64_t p) -> uint32_t {
    uint32_t v = __ldcg(a.key + p);
    if (a.key_packed) v &= 0xffffu;
    return v - a.key_base;
  };
  for (int64_t p = p0 + lane; p < p1; p += 32) {
    const uint32_t e = key(p);
    if (e < (uint32_t)E) atomicAdd(&wcnt[warp * E + e], 1);
  }
  __syncthreads();
  // experts e = c*128 + tid, in chunks of 128 (expert order = chunk, then thread)
  int32_t base_carry = 0, act_carry = 0, tile_carry = 0;
  for (int c = 0; c * 128 < E; ++c) {
    const int e = c * 128 + tid;
    int32_t tot = 0;
    if (e < E) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const int32_t h = wcnt[w * E + e];
        wcnt[w * E + e] = tot;
        tot += h;
      }
    }
    int32_t ctot, cact, ctile;
    const int32_t base = base_carry + scan128(e < E ? tot : 0, sh, &ctot);
    const int32_t arank = act_carry + scan128((e < E && tot > 0) ? 1 : 0, sh, &cact);
    const int32_t nt = (e < E && tot >= a.tc_min_rows) ? (tot + a.tile_rows - 1) / a.tile_rows : 0;
    const int32_t tb = tile_carry + scan128(nt, sh, &ctile);
    if (e < E) {
      a.offsets[e] = base;
      if (tot > 0) a.active[arank] = e;
      if (a.tile_start) a.tile_start[e] = tb;
#pragma unroll
      for (int w = 0; w < 4; ++w) wcnt[w * E + e] += base;
    }
    base_carry += ctot;
    act_carry += cact;
    tile_carry += ctile;
  }
  if (tid == 0) {
    a.offsets[E] = base_carry;
    *a.n_active = act_carry;
    if (a.tile_start) a.tile_start[E] = tile_carry;
  }
  __syncthreads();
  int32_t* cur = wcnt + warp * E;
  for (int64_t b = p0; b < p1; b += 32) {
    const int64_t p = b + lane;
    const bool valid = p < p1;
    const uint32_t e = valid ? key(p) : 0xffffffffu;
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const unsigned lt = (1u << lane) - 1u;
    int32_t pos = 0;
    if (valid && e < (uint32_t)E) {
      pos = cur[e] + __popc(peers & lt);
      a.perm[pos] = (uint32_t)p;
      if (a.inv) a.inv[p] = (uint32_t)pos;
    }
    __syncwarp();
    if (valid && e < (uint32_t)E && (peers >> lane) == 1u) cur[e] = pos + 1;
    __syncwarp();
  }
}

// Grid (row tiles of 4*NE rows, token tiles of NT tokens), 128 threads. counters:
// [0, gridDim.y) per token tile, [gridDim.y] global. Dynamic shared memory: 4 * E ints.
template <int NE, int NT, int PL>
__global__ void __launch_bounds__(128) route_fused_kernel(RouterArgs ra, TopkArgs ta, GroupArgs ga, int do_group,
                                                          uint32_t* counters) {
  extern __shared__ int32_t wcnt[];
  __shared__ int32_t sh[4];
  __shared__ uint32_t ticket;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.y * NT;
  pdl_wait();
  // no early launch_dependents: the next kernel's CTAs (the GEMV: 512 threads, ~200 KB of
  // shared memory) would wait resident on the SMs this kernel's later CTAs need (measured:
  // a Qwen3 T=64 block 167.9 us with the early trigger, 157.7 us without); every CTA's
  // exit counts as its trigger
  router_tile<NE, NT>(ra, (blockIdx.x * 4 + warp) * NE, t0, lane);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) ticket = atomicAdd(&counters[blockIdx.y], 1u);
  __syncthreads();
  if (ticket != gridDim.x - 1) return;  // not the last CTA of this token tile
  __threadfence();
  if (warp < NT && t0 + warp < ta.T) topk_token<PL>(ta, t0 + warp, lane);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    counters[blockIdx.y] = 0;
    ticket = do_group ? atomicAdd(&counters[gridDim.y], 1u) : 0u;
  }
  __syncthreads();
  if (!do_group || ticket != gridDim.y - 1) return;  // not the last token tile
  __threadfence();
  group_cta128(ga, wcnt, sh);
  if (threadIdx.x == 0) counters[gridDim.y] = 0;
}

template <int NE, int NT>
static cudaError_t launch_fused_t(const RouterArgs& ra, const TopkArgs& ta, const GroupArgs* ga,
                                  uint32_t* counters, cudaStream_t st) {
  dim3 grid((ra.n_rows + 4 * NE - 1) / (4 * NE), (ra.T + NT - 1) / NT);
  const GroupArgs g = ga ? *ga : GroupArgs{};
  const size_t smem = ga ? sizeof(int32_t) * 4 * (size_t)ga->E : 0;
  const int pl = (ta.E + 31) / 32, dg = ga ? 1 : 0;
  if (pl <= 1) return launch_k(route_fused_kernel<NE, NT, 1>, grid, dim3(128), smem, st, ra, ta, g, dg, counters);
  if (pl <= 2) return launch_k(route_fused_kernel<NE, NT, 2>, grid, dim3(128), smem, st, ra, ta, g, dg, counters);
  if (pl <= 4) return launch_k(route_fused_kernel<NE, NT, 4>, grid, dim3(128), smem, st, ra, ta, g, dg, counters);
  if (pl <= 8) return launch_k(route_fused_kernel<NE, NT, 8>, grid, dim3(128), smem, st, ra, ta, g, dg, counters);
  return launch_k(route_fused_kernel<NE, NT, 16>, grid, dim3(128), smem, st, ra, ta, g, dg, counters);
}

bool route_fused_fits(int T, int E, int64_t P) {
  return T >= 1 && T <= kFusedRouteMaxTokens && E <= 512 && P <= 4096;
}

cudaError_t launch_route_fused(const RouterArgs& ra, const TopkArgs& ta, const GroupArgs* ga, uint32_t* counters,
                               cudaStream_t st) {
  if (ra.T <= 4) return launch_fused_t<1, 1>(ra, ta, ga, counters, st);
  return launch_fused_t<2, 4>(ra, ta, ga, counters, st);
}

cudaError_t launch_router(const RouterArgs& a, cudaStream_t st) {
  if (a.T <= 0) return cudaSuccess;
  if (a.xf) {  // f32 token rows, f32 logits
    if (a.T <= 4) return launch_k(router_logits_f32_kernel<1, 1>, dim3((a.n_rows + 3) / 4, a.T), dim3(128), 0, st, a);
    return launch_k(router_logits_f32_kernel<2, 4>, dim3((a.n_rows + 7) / 8, (a.T + 3) / 4), dim3(128), 0, st, a);
  }
  if (a.T <= 4) {
    dim3 grid((a.n_rows + 3) / 4, a.T);
    return launch_k(router_logits_kernel<1, 1>, grid, dim3(128), 0, st, a);
  } else if (a.T <= 64) {
    dim3 grid((a.n_rows + 7) / 8, (a.T + 3) / 4);
    return launch_k(router_logits_kernel<2, 4>, grid, dim3(128), 0, st, a);
  }
  // large batches: the token rows staged once per CTA in shared memory as f32 pairs
  // (KMAX * 32 bytes); as many warps (at most 8) as spread the row groups evenly.
  // Measured on the B200 (Qwen3-30B-A3B router, 128 x 2048): T=4096 100.7 us against
  // 131.9 us for router_logits_kernel<4, 8>, T=1024 46.9 against 49.3; at T=72 the
  // latter is faster (27.0 against 36.1 us).
  if (a.T >= 128 && a.K <= 2048 && a.K % 64 == 0) {
    constexpr size_t smem = (size_t)(kRsTok / 2) * 2048 * 8;
    static thread_local int set_dev = -1;
    static thread_local int nsm = 0;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return err;
    if (dev != set_dev) {
      err = cudaFuncSetAttribute(router_logits_smem_kernel<2048>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (err != cudaSuccess) return err;
      err = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
      if (err != cudaSuccess) return err;
      set_dev = dev;
    }
    const int ngroups = (a.n_rows + kRsRowsPerWarp - 1) / kRsRowsPerWarp;
    const int ntg = (a.T + kRsTok - 1) / kRsTok;
    // split the rows while the CTAs (8 tokens each) are fewer than 4 per SM, keeping at
    // least 4 row groups (4 warps) per CTA
    int splits = 1;
    while (2 * splits * 4 <= ngroups && (long)ntg * splits < 4L * nsm) splits *= 2;
    const int gpc = (ngroups + splits - 1) / splits;
    const int per_warp = (gpc + kRsMaxWarps - 1) / kRsMaxWarps;
    const int nwarps = (gpc + per_warp - 1) / per_warp;
    return launch_k(router_logits_smem_kernel<2048>, dim3(ntg, splits), dim3(nwarps * 32), smem, st, a);
  }
  dim3 grid((a.n_rows + 15) / 16, (a.T + 7) / 8);
  return launch_k(router_logits_kernel<4, 8>, grid, dim3(128), 0, st, a);
}

cudaError_t launch_topk(const TopkArgs& a, cudaStream_t st) {
  if (a.T <= 0) return cudaSuccess;
  const int blocks = (a.T + 3) / 4;
  const int pl = (a.E + 31) / 32;
  if (pl <= 1) return launch_k(topk_kernel<1>, dim3(blocks), dim3(128), 0, st, a);
  if (pl <= 2) return launch_k(topk_kernel<2>, dim3(blocks), dim3(128), 0, st, a);
  if (pl <= 4) return launch_k(topk_kernel<4>, dim3(blocks), dim3(128), 0, st, a);
  if (pl <= 8) return launch_k(topk_kernel<8>, dim3(blocks), dim3(128), 0, st, a);
  return launch_k(topk_kernel<16>, dim3(blocks), dim3(128), 0, st, a);
}

}  // namespace moe
