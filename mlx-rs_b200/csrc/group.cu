// group.cu — deterministic counting sort of (token, slot) pairs by expert.
//
// MLX's gather_qmm groups rows by expert internally when sorted_indices=false
// (SwitchLinear::forward, qwen3_moe_python_port.rs:311-324); here the grouping is an
// explicit, stable counting sort so that the per-expert row lists are reproducible
// bit for bit: offsets[e] = exclusive prefix sum of the counts, and within expert e
// the pairs p = t*k + j appear in ascending p.
//
// Small inputs (P <= 8192, E <= 512) take one launch of one CTA (group_small_kernel):
// 32 warps each own a contiguous segment of the pairs; per-warp histograms in shared
// memory give every warp its per-expert base, and each warp then ranks its pairs in
// order with __match_any_sync. Larger inputs take three launches over segments of
// `seg` consecutive pairs:
//   hist:    per-segment histograms (shared-memory atomics; counts are order-free);
//   scan:    one CTA: per-expert prefix over segments (histogram staged in shared
//            memory), exclusive scan over experts, the ascending list of active experts;
//   scatter: one warp per segment walks its pairs in order, 32 at a time; lanes with
//            the same expert are ranked by __match_any_sync, so positions follow p.
#include "common.cuh"
#include "kernels.cuh"

namespace moe {

MOE_DEV uint32_t group_key(const GroupArgs& a, int64_t p) {
  uint32_t v = a.key[p];
  if (a.key_packed) v &= 0xffffu;
  return v - a.key_base;
}

// Block-wide exclusive scan of one value per thread (thread order); returns the
// exclusive prefix and writes the total to *total (1024 threads).
MOE_DEV int32_t block_exclusive_scan(int32_t v, int32_t* warp_tot, int32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int32_t u = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += u;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int32_t w = warp_tot[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int32_t u = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += u;
    }
    warp_tot[lane] = w;
  }
  __syncthreads();
  const int32_t excl = incl - v + (warp > 0 ? warp_tot[warp - 1] : 0);
  if (total) *total = warp_tot[31];
  __syncthreads();
  return excl;
}

// One CTA of 1024 threads. Shared memory: wbase[32][E] per-warp counts, then bases.
__global__ void __launch_bounds__(1024) group_small_kernel(GroupArgs a) {
  extern __shared__ int32_t wbase[];
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t n_act;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int E = a.E;
  pdl_wait();
  for (int i = tid; i < 32 * E; i += 1024) wbase[i] = 0;
  __syncthreads();
  const int64_t seg = (a.P + 31) / 32;
  const int64_t p0 = warp * seg;
  const int64_t p1 = (p0 + seg < a.P) ? p0 + seg : a.P;
  // the warp's keys stay in registers for the scatter below (P <= 8192: at most 8 rounds
  // of 32 pairs per warp), all loads issued before the first is used
  constexpr int kRounds = 8;
  uint32_t keys[kRounds];
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int64_t p = p0 + r * 32 + lane;
    keys[r] = p < p1 ? group_key(a, p) : 0xffffffffu;
  }
#pragma unroll
  for (int r = 0; r < kRounds; ++r)
    if (keys[r] < (uint32_t)E) atomicAdd(&wbase[warp * E + keys[r]], 1);
  __syncthreads();
  // per expert (thread e): prefix over warps; expert totals
  int32_t tot = 0;
  if (tid < E) {
    for (int w = 0; w < 32; ++w) {
      const int32_t h = wbase[w * E + tid];
      wbase[w * E + tid] = tot;
      tot += h;
    }
  }
  const int32_t base = block_exclusive_scan(tid < E ? tot : 0, warp_tot, nullptr);
  const int32_t arank = block_exclusive_scan((tid < E && tot > 0) ? 1 : 0, warp_tot, &n_act);
  if (a.tile_start) {
    const int32_t nt = (tid < E && tot >= a.tc_min_rows) ? (tot + a.tile_rows - 1) / a.tile_rows : 0;
    const int32_t tbase = block_exclusive_scan(nt, warp_tot, nullptr);
    if (tid <= E) a.tile_start[tid] = tbase;
  }
  if (tid < E) {
    a.offsets[tid] = base;
    if (tot > 0) a.active[arank] = tid;
    for (int w = 0; w < 32; ++w) wbase[w * E + tid] += base;
  }
  if (tid == E) a.offsets[E] = base;  // thread E holds the exclusive total of experts 0..E-1
  if (tid == 0) *a.n_active = n_act;
  pdl_trigger();
  __syncthreads();
  // stable scatter: warp w walks its segment in order, 32 pairs at a time
  int32_t* cur = wbase + warp * E;
#pragma unroll
  for (int r = 0; r < kRounds; ++r) {
    const int64_t b = p0 + r * 32;
    if (b >= p1) break;
    const int64_t p = b + lane;
    const bool valid = p < p1;
    const uint32_t e = keys[r];
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

__global__ void group_hist_kernel(GroupArgs a) {
  extern __shared__ int32_t sh[];
  const int g = blockIdx.x;
  pdl_wait();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int64_t p0 = (int64_t)g * a.seg;
  const int64_t p1 = (p0 + a.seg < a.P) ? p0 + a.seg : a.P;
  for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
    const uint32_t e = group_key(a, p);
    if (e < (uint32_t)a.E) atomicAdd(&sh[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) a.hist[(size_t)g * a.E + e] = sh[e];
}

// One CTA of 1024 threads (E <= 4096). The [nseg, E] histogram is staged in shared memory
// (nseg * E * 4 bytes, sized by the caller's choice of segment length); the per-expert
// prefix over segments runs on several threads per expert (runs of segments, then a
// shuffle scan of the runs' sums), and for the scan over experts thread t owns experts
// 4t .. 4t+3; the results go back to global memory coalesced.
__global__ void __launch_bounds__(1024) group_scan_kernel(GroupArgs a) {
  extern __shared__ int32_t hs[];  // [nseg][E]
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t n_act;
  __shared__ int32_t etot_s[4096];  // per-expert totals, later per-expert bases (E <= 4096)
  constexpr int EPT = 4;
  const int tid = threadIdx.x;
  const int E = a.E;
  const int n = a.nseg * E;
  pdl_wait();
  // 8 loads in flight per thread, then their stores (one CTA moves the whole histogram)
  for (int i0 = 0; i0 < n; i0 += 8 * 1024) {
    int32_t v[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int i = i0 + r * 1024 + tid;
      v[r] = i < n ? __ldcg(a.hist + i) : 0;
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int i = i0 + r * 1024 + tid;
      if (i < n) hs[i] = v[r];
    }
  }
  __syncthreads();
  // per-expert exclusive prefix over the segments, in place: tpe threads per expert (a
  // power of two, 1024 / E rounded down, 1 to 32), thread j of an expert owns a run of
  // consecutive segments; the runs' sums are scanned across the tpe lanes with shuffles
  int tpe = 1;
  while (tpe < 32 && tpe * 2 * E <= 1024) tpe *= 2;
  const int eper = 1024 / tpe;  // experts per pass
  const int cs = (a.nseg + tpe - 1) / tpe;
  const int j = tid % tpe;
  for (int e0 = 0; e0 < E; e0 += eper) {
    const int e = e0 + tid / tpe;
    const bool ev = e < E;
    const int g0 = j * cs, g1 = (g0 + cs < a.nseg) ? g0 + cs : a.nseg;
    int32_t local = 0;
    if (ev)
      for (int g = g0; g < g1; ++g) local += hs[g * E + e];
    int32_t incl = local;
    for (int off = 1; off < tpe; off <<= 1) {
      const int32_t u = __shfl_up_sync(0xffffffffu, incl, off, tpe);
      if (j >= off) incl += u;
    }
    const int32_t etotal = __shfl_sync(0xffffffffu, incl, tpe - 1, tpe);
    if (ev) {
      int32_t run = incl - local;
      for (int g = g0; g < g1; ++g) {
        const int32_t h = hs[g * E + e];
        hs[g * E + e] = run;
        run += h;
      }
      if (j == 0) etot_s[e] = etotal;
    }
  }
  __syncthreads();
  int32_t tot[EPT];
  int32_t my_sum = 0, my_act = 0;
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const int e = tid * EPT + i;
    const int32_t run = e < E ? etot_s[e] : 0;
    tot[i] = run;    my_sum += run;
    my_act += run > 0 ? 1 : 0;
  }
  const int32_t base0 = block_exclusive_scan(my_sum, warp_tot, nullptr);
  const int32_t abase0 = block_exclusive_scan(my_act, warp_tot, &n_act);
  int32_t base = base0, abase = abase0;
  int32_t ebase[EPT];
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const int e = tid * EPT + i;
    ebase[i] = base;
    if (e < E) {
      a.offsets[e] = base;
      if (tot[i] > 0) a.active[abase++] = e;
      base += tot[i];
    }
  }
  if (tid * EPT < E && (tid + 1) * EPT >= E) a.offsets[E] = base;  // total of valid pairs
  if (tid == 0) *a.n_active = n_act;
  if (a.tile_start) {
    int32_t nt[EPT], my_nt = 0;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      nt[i] = (tid * EPT + i < E && tot[i] >= a.tc_min_rows) ? (tot[i] + a.tile_rows - 1) / a.tile_rows : 0;
      my_nt += nt[i];
    }
    int32_t tb = block_exclusive_scan(my_nt, warp_tot, nullptr);
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      const int e = tid * EPT + i;
      if (e <= E) a.tile_start[e] = tb;  // entry E (the total) from the thread past the last expert
      tb += nt[i];
    }
  }
  // segment bases -> global memory, each plus its expert's base (coalesced over the
  // [nseg, E] layout; the expert bases go through shared memory)
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const int e = tid * EPT + i;
    if (e < E) etot_s[e] = ebase[i];
  }
  __syncthreads();
  for (int i = tid; i < n; i += 1024) a.segbase[i] = hs[i] + etot_s[i % E];
}

__global__ void group_scatter_kernel(GroupArgs a) {
  extern __shared__ int32_t cur[];
  const int g = blockIdx.x;
  const int lane = threadIdx.x;
  pdl_wait();
  for (int e = lane; e < a.E; e += 32) cur[e] = a.segbase[(size_t)g * a.E + e];
  __syncwarp();
  const int64_t p0 = (int64_t)g * a.seg;
  const int64_t p1 = (p0 + a.seg < a.P) ? p0 + a.seg : a.P;
  constexpr int kRounds = 8;  // keys of this many rounds of 32 pairs loaded before the first is ranked
  for (int64_t chunk = p0; chunk < p1; chunk += 32 * kRounds) {
    uint32_t keys[kRounds];
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int64_t p = chunk + r * 32 + lane;
      keys[r] = p < p1 ? group_key(a, p) : 0xffffffffu;
    }
#pragma unroll
    for (int r = 0; r < kRounds; ++r) {
      const int64_t base = chunk + r * 32;
      if (base >= p1) break;
      const int64_t p = base + lane;
      const bool valid = p < p1;
      const uint32_t e = keys[r];
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      const unsigned lt = (1u << lane) - 1u;
      int32_t pos = 0;
      if (valid && e < (uint32_t)a.E) {
        pos = cur[e] + __popc(peers & lt);
        a.perm[pos] = (uint32_t)p;
        if (a.inv) a.inv[p] = (uint32_t)pos;
      }
      __syncwarp();
      // The highest lane of each group of equal experts advances the cursor.
      if (valid && e < (uint32_t)a.E && (peers >> lane) == 1u) cur[e] = pos + 1;
      __syncwarp();
    }
  }
}

cudaError_t launch_group(const GroupArgs& a, cudaStream_t st) {
  if (a.P <= 0) {
    // Empty input: offsets all zero, no active experts.
    cudaError_t err = cudaMemsetAsync(a.offsets, 0, sizeof(int32_t) * (a.E + 1), st);
    if (err != cudaSuccess) return err;
    return cudaMemsetAsync(a.n_active, 0, sizeof(int32_t), st);
  }
  if (a.P <= 8192 && a.E <= 512) {  // 8 rounds of 32 pairs per warp of group_small_kernel at most
    const size_t smem = sizeof(int32_t) * 32 * a.E;
    static thread_local int set_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != set_dev) {
      cudaError_t err = cudaFuncSetAttribute(group_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)(sizeof(int32_t) * 32 * 512));
      if (err != cudaSuccess) return err;
      set_dev = dev;
    }
    return launch_k(group_small_kernel, dim3(1), dim3(1024), smem, st, a);
  }
  const size_t sh = sizeof(int32_t) * a.E;
  const size_t scan_sh = sizeof(int32_t) * (size_t)a.nseg * a.E;
  if (scan_sh > kGroupScanSmem) return cudaErrorInvalidValue;  // the caller's segment length is too short
  {
    static thread_local int set_dev = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev != set_dev) {
      cudaError_t err = cudaFuncSetAttribute(group_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kGroupScanSmem);
      if (err != cudaSuccess) return err;
      set_dev = dev;
    }
  }
  cudaError_t err = launch_k(group_hist_kernel, dim3(a.nseg), dim3(256), sh, st, a);
  if (err != cudaSuccess) return err;
  err = launch_k(group_scan_kernel, dim3(1), dim3(1024), scan_sh, st, a);
  if (err != cudaSuccess) return err;
  return launch_k(group_scatter_kernel, dim3(a.nseg), dim3(32), sh, st, a);
}

}  // namespace moe
