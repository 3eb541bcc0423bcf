// ep.cu — the two kernels that expert parallelism adds around the block's kernels.
//
// Under expert parallelism rank r owns experts [e0, e0 + E_l) of every block and the
// tokens [r*T_l, (r+1)*T_l). The token rows are all-gathered, every rank routes all of
// them (packed routing: expert | bf16 weight << 16), runs its experts over the pairs that
// selected them, and the per-token partial sums travel back
// to the token's owner with an all-to-all, where they are added in rank order.
//
// ep_partial: the combine of SparseMoeBlock::forward (expert_out * score, sum_axis(1),
//   qwen3_moe_python_port.rs:471-472; lfm2_moe_python_port.rs:718-732) restricted to
//   the local experts: partial[t] = sum over j = 0..k-1 in index order, of the local
//   pairs only, of bf16(y * w_j), in fp32 and not rounded (the owner rounds once), or
//   rounded once to bf16 (half the bytes through the combine's all-to-all; the owner's
//   sum then adds bf16-rounded partials).
//   Each thread owns 8 consecutive hidden elements of one token, as in combine.cu.
// ep_finish: out[t] = bf16(sum over ranks s in order of partial_s[t]) (fp32 or bf16
//   partials, summed in fp32); optionally the
//   next block's RMSNorm (RmsNorm::forward, crates/mlx-nn/src/rms_norm.rs:30-34) of
//   out in the same pass, with the canonical sum of squares of rms_norm_kernel.
#include "common.cuh"
#include "kernels.cuh"

namespace moe {

__global__ void __launch_bounds__(256) ep_partial_kernel(EpPartialArgs a) {
  const int vec_per_row = a.H >> 3;
  const int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  pdl_wait();
  pdl_trigger();
  if (id >= (int64_t)a.T * vec_per_row) return;
  const int t = (int)(id / vec_per_row);
  const int h = (int)(id - (int64_t)t * vec_per_row) * 8;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  // k terms in batches of 4 with their loads in flight together, summed in index order
  for (int j0 = 0; j0 < a.k; j0 += 4) {
    uint4 v[4];
    float wj[4];
    bool loc[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = j0 + jj;
      loc[jj] = false;
      if (j < a.k) {
        const int64_t p = (int64_t)t * a.k + j;
        const uint32_t pk = a.packed[p];
        loc[jj] = (pk & 0xffffu) - a.e0 < (uint32_t)a.E_l;  // else another rank's expert
        if (loc[jj]) {
          wj[jj] = bf2f((uint16_t)(pk >> 16));
          v[jj] = *reinterpret_cast<const uint4*>(a.y + (size_t)a.inv[p] * a.H + h);
        }
      }
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      if (loc[jj]) {
        const uint32_t u[4] = {v[jj].x, v[jj].y, v[jj].z, v[jj].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[2 * i] = __fadd_rn(acc[2 * i], rbf(__fmul_rn(bf_lo(u[i]), wj[jj])));
          acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], rbf(__fmul_rn(bf_hi(u[i]), wj[jj])));
        }
      }
    }
  }
  if (a.partial_bf16) {
    uint4 o;
    o.x = (uint32_t)f2bf(acc[0]) | ((uint32_t)f2bf(acc[1]) << 16);
    o.y = (uint32_t)f2bf(acc[2]) | ((uint32_t)f2bf(acc[3]) << 16);
    o.z = (uint32_t)f2bf(acc[4]) | ((uint32_t)f2bf(acc[5]) << 16);
    o.w = (uint32_t)f2bf(acc[6]) | ((uint32_t)f2bf(acc[7]) << 16);
    *reinterpret_cast<uint4*>(a.partial_bf16 + (size_t)t * a.H + h) = o;
    return;
  }
  float4* dst = reinterpret_cast<float4*>(a.partial + (size_t)t * a.H + h);
  dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

// 8 consecutive partial values of one rank as fp32 (bf16 partials widen exactly).
MOE_DEV void load8(const float* p, float (&v)[8]) {
  const float4 x0 = reinterpret_cast<const float4*>(p)[0], x1 = reinterpret_cast<const float4*>(p)[1];
  v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
  v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
}
MOE_DEV void load8(const uint16_t* p, float (&v)[8]) {
  const uint4 x = *reinterpret_cast<const uint4*>(p);
  v[0] = bf_lo(x.x); v[1] = bf_hi(x.x); v[2] = bf_lo(x.y); v[3] = bf_hi(x.y);
  v[4] = bf_lo(x.z); v[5] = bf_hi(x.z); v[6] = bf_lo(x.w); v[7] = bf_hi(x.w);
}

// One warp per row; lane l owns the chunks of 8 elements c = l, l + 32, ... Partials in
// fp32 or bf16 (PT).
template <class PT>
__global__ void __launch_bounds__(256) ep_finish_kernel(const PT* __restrict__ recv, int world, int64_t rows,
                                                        int H, uint16_t* __restrict__ out,
                                                        const uint16_t* __restrict__ norm_w, float eps,
                                                        uint16_t* __restrict__ normed) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  pdl_wait();
  pdl_trigger();
  if (r >= rows) return;
  const int nchunks = H >> 3;
  const size_t rank_stride = (size_t)rows * H;
  float ss = 0.0f;
  for (int c = lane; c < nchunks; c += 32) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.0f;
    for (int s = 0; s < world; ++s) {
      float x[8];
      load8(recv + s * rank_stride + (size_t)r * H + c * 8, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __fadd_rn(v[i], x[i]);
    }
    uint16_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i] = f2bf(v[i]);
      const float q = bf2f(o[i]);
      ss = __fmaf_rn(q, q, ss);
    }
    uint4 ov;
    ov.x = (uint32_t)o[0] | ((uint32_t)o[1] << 16);
    ov.y = (uint32_t)o[2] | ((uint32_t)o[3] << 16);
    ov.z = (uint32_t)o[4] | ((uint32_t)o[5] << 16);
    ov.w = (uint32_t)o[6] | ((uint32_t)o[7] << 16);
    *reinterpret_cast<uint4*>(out + (size_t)r * H + c * 8) = ov;
  }
  if (!norm_w) return;
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, off));
  const float rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), eps)));
  for (int c = lane; c < nchunks; c += 32) {
    // this thread's own stores above
    const uint4 v = *reinterpret_cast<const uint4*>(out + (size_t)r * H + c * 8);
    const uint4 wv = *reinterpret_cast<const uint4*>(norm_w + c * 8);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint16_t lo = f2bf(__fmul_rn(rbf(__fmul_rn(bf_lo(u[i]), rr)), bf_lo(wu[i])));
      const uint16_t hi = f2bf(__fmul_rn(rbf(__fmul_rn(bf_hi(u[i]), rr)), bf_hi(wu[i])));
      o[i] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint4*>(normed + (size_t)r * H + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

cudaError_t launch_ep_partial(const EpPartialArgs& a, cudaStream_t st) {
  const int64_t n = (int64_t)a.T * (a.H >> 3);
  if (n <= 0) return cudaSuccess;
  return launch_k(ep_partial_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, a);
}

cudaError_t launch_ep_finish(const float* recv, int world, int64_t rows, int H, uint16_t* out,
                             const uint16_t* norm_w, float eps, uint16_t* normed, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  return launch_k(ep_finish_kernel<float>, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, st, recv, world, rows, H,
                  out, norm_w, eps, normed);
}

cudaError_t launch_ep_finish_bf16(const uint16_t* recv, int world, int64_t rows, int H, uint16_t* out,
                                  const uint16_t* norm_w, float eps, uint16_t* normed, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  return launch_k(ep_finish_kernel<uint16_t>, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, st, recv, world, rows,
                  H, out, norm_w, eps, normed);
}

}  // namespace moe
