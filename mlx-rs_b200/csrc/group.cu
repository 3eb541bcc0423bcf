// group.cu — deterministic counting sort of (token, slot) pairs by expert.
//
// MLX's gather_qmm groups rows by expert internally when sorted_indices=false
// (SwitchLinear::forward, qwen3_moe_python_port.rs:311-324); here the grouping is an
// explicit, stable counting sort so that the per-expert row lists are reproducible
// bit for bit: offsets[e] = exclusive prefix sum of the counts, and within expert e
// the pairs p = t*k + j appear in ascending p.
//
// Three launches over segments of `seg` consecutive pairs:
//   hist:    per-segment histograms (shared-memory atomics; counts are order-free);
//   scan:    one CTA: per-expert prefix over segments, exclusive scan over experts,
//            the ascending list of active experts;
//   scatter: one warp per segment walks its pairs in order, 32 at a time; lanes with
//            the same expert are ranked by __match_any_sync, so positions follow p.
#include "common.cuh"
#include "kernels.cuh"

namespace moe {

__global__ void group_hist_kernel(GroupArgs a) {
  extern __shared__ int32_t sh[];
  const int g = blockIdx.x;
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) sh[e] = 0;
  __syncthreads();
  const int64_t p0 = (int64_t)g * a.seg;
  const int64_t p1 = (p0 + a.seg < a.P) ? p0 + a.seg : a.P;
  for (int64_t p = p0 + threadIdx.x; p < p1; p += blockDim.x) {
    const uint32_t e = a.key[p];
    if (e < (uint32_t)a.E) atomicAdd(&sh[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) a.hist[(size_t)g * a.E + e] = sh[e];
}

// One CTA of 1024 threads; thread t owns experts 4t .. 4t+3 (E <= 4096).
__global__ void __launch_bounds__(1024) group_scan_kernel(GroupArgs a) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t warp_act[32];
  constexpr int EPT = 4;
  const int tid = threadIdx.x;
  int32_t tot[EPT];
  int32_t my_sum = 0, my_act = 0;
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const int e = tid * EPT + i;
    int32_t run = 0;
    if (e < a.E) {
      for (int g = 0; g < a.nseg; ++g) {
        const int32_t h = a.hist[(size_t)g * a.E + e];
        a.segbase[(size_t)g * a.E + e] = run;
        run += h;
      }
    }
    tot[i] = run;
    my_sum += run;
    my_act += run > 0 ? 1 : 0;
  }
  // Block-wide exclusive scan of my_sum and my_act (thread order = expert order).
  const int lane = tid & 31, warp = tid >> 5;
  int32_t incl = my_sum, incl_a = my_act;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int32_t v = __shfl_up_sync(0xffffffffu, incl, off);
    const int32_t va = __shfl_up_sync(0xffffffffu, incl_a, off);
    if (lane >= off) {
      incl += v;
      incl_a += va;
    }
  }
  if (lane == 31) {
    warp_tot[warp] = incl;
    warp_act[warp] = incl_a;
  }
  __syncthreads();
  if (warp == 0) {
    int32_t v = warp_tot[lane], va = warp_act[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int32_t u = __shfl_up_sync(0xffffffffu, v, off);
      const int32_t ua = __shfl_up_sync(0xffffffffu, va, off);
      if (lane >= off) {
        v += u;
        va += ua;
      }
    }
    warp_tot[lane] = v;
    warp_act[lane] = va;
  }
  __syncthreads();
  int32_t base = incl - my_sum + (warp > 0 ? warp_tot[warp - 1] : 0);
  int32_t abase = incl_a - my_act + (warp > 0 ? warp_act[warp - 1] : 0);
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const int e = tid * EPT + i;
    if (e < a.E) {
      a.offsets[e] = base;
      for (int g = 0; g < a.nseg; ++g) a.segbase[(size_t)g * a.E + e] += base;
      if (tot[i] > 0) a.active[abase++] = e;
      base += tot[i];
    }
  }
  if (tid == 0) {
    a.offsets[a.E] = (int32_t)a.P;
    *a.n_active = warp_act[31];
  }
}

__global__ void group_scatter_kernel(GroupArgs a) {
  extern __shared__ int32_t cur[];
  const int g = blockIdx.x;
  const int lane = threadIdx.x;
  for (int e = lane; e < a.E; e += 32) cur[e] = a.segbase[(size_t)g * a.E + e];
  __syncwarp();
  const int64_t p0 = (int64_t)g * a.seg;
  const int64_t p1 = (p0 + a.seg < a.P) ? p0 + a.seg : a.P;
  for (int64_t base = p0; base < p1; base += 32) {
    const int64_t p = base + lane;
    const bool valid = p < p1;
    const uint32_t e = valid ? a.key[p] : 0xffffffffu;
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

cudaError_t launch_group(const GroupArgs& a, cudaStream_t st) {
  if (a.P <= 0) {
    // Empty input: offsets all zero, no active experts.
    cudaError_t err = cudaMemsetAsync(a.offsets, 0, sizeof(int32_t) * (a.E + 1), st);
    if (err != cudaSuccess) return err;
    return cudaMemsetAsync(a.n_active, 0, sizeof(int32_t), st);
  }
  const size_t sh = sizeof(int32_t) * a.E;
  group_hist_kernel<<<a.nseg, 256, sh, st>>>(a);
  group_scan_kernel<<<1, 1024, 0, st>>>(a);
  group_scatter_kernel<<<a.nseg, 32, sh, st>>>(a);
  return cudaGetLastError();
}

}  // namespace moe
