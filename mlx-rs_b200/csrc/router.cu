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
  pdl_trigger();
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
