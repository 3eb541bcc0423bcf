// combine.cu — weighted combine of the k expert outputs (+ gated shared expert) and RMSNorm.
//
// combine: out[t] = bf16( sum_j bf16(y[t,j] * w[t,j]) ), fp32 sum over j = 0..k-1 in
// index order (expert_out.multiply(score).sum_axis(1), qwen3_moe_python_port.rs:471-472;
// lfm2_moe_python_port.rs:718-732), then, with a shared expert,
// out = bf16(out + bf16(shared * bf16(sigmoid(gate_logit)))) (:477-484).
// With a residual (the decoder layer's FFN half), out = bf16(residual + out) last:
// residual.add(ff.forward(h)), qwen3_moe_python_port.rs:736-739 and
// lfm2_moe_python_port.rs:856-868.
// Each thread owns 8 consecutive hidden elements of one token (16-byte loads/stores).
//
// rms_norm: y = bf16(bf16(x * r) * w), r = 1 / sqrt(sum(x^2) / dim + eps) with IEEE
// sqrt and divide; sum(x^2) in the canonical order (lane l of a warp owns the chunks
// of 8 elements c = l, l+32, ..., fma per element, then the xor butterfly), which the
// CPU oracle evaluates identically. RmsNorm::forward, crates/mlx-nn/src/rms_norm.rs:30-34.
#include "common.cuh"
#include "kernels.cuh"

namespace moe {

__global__ void __launch_bounds__(256) combine_kernel(CombineArgs a) {
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
  // k terms in batches of 4: the row indices, weights and rows of a batch are loaded
  // before any is used (independent loads in flight), then summed in index order.
  for (int j0 = 0; j0 < a.k; j0 += 4) {
    uint4 v[4];
    float wj[4];
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = j0 + jj;
      if (j < a.k) {
        const int64_t p = (int64_t)t * a.k + j;
        wj[jj] = bf2f(a.weights[p]);
        v[jj] = *reinterpret_cast<const uint4*>(a.y + (size_t)a.inv[p] * a.H + h);
      }
    }
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      if (j0 + jj < a.k) {
        const uint32_t u[4] = {v[jj].x, v[jj].y, v[jj].z, v[jj].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[2 * i] = __fadd_rn(acc[2 * i], rbf(__fmul_rn(bf_lo(u[i]), wj[jj])));
          acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], rbf(__fmul_rn(bf_hi(u[i]), wj[jj])));
        }
      }
    }
  }
  uint16_t o[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i] = f2bf(acc[i]);
  if (a.shared) {
    const uint4 v = *reinterpret_cast<const uint4*>(a.shared + (size_t)t * a.H + h);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    const bool gated = a.gate_val != nullptr;
    const float gv = gated ? bf2f(a.gate_val[t]) : 1.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float s = (i & 1) ? bf_hi(u[i >> 1]) : bf_lo(u[i >> 1]);
      if (gated) s = rbf(__fmul_rn(s, gv));
      o[i] = f2bf(__fadd_rn(bf2f(o[i]), s));
    }
  }
  if (a.residual) {
    const uint4 v = *reinterpret_cast<const uint4*>(a.residual + (size_t)t * a.H + h);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float r = (i & 1) ? bf_hi(u[i >> 1]) : bf_lo(u[i >> 1]);
      o[i] = f2bf(__fadd_rn(r, bf2f(o[i])));
    }
  }
  uint4 ov;
  ov.x = (uint32_t)o[0] | ((uint32_t)o[1] << 16);
  ov.y = (uint32_t)o[2] | ((uint32_t)o[3] << 16);
  ov.z = (uint32_t)o[4] | ((uint32_t)o[5] << 16);
  ov.w = (uint32_t)o[6] | ((uint32_t)o[7] << 16);
  *reinterpret_cast<uint4*>(a.out + (size_t)t * a.H + h) = ov;
}

__global__ void __launch_bounds__(256) rms_norm_kernel(const uint16_t* __restrict__ x,
                                                       const uint16_t* __restrict__ w, float eps,
                                                       int64_t rows, int dim, uint16_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  pdl_wait();
  pdl_trigger();
  if (r >= rows) return;
  const uint16_t* xr = x + (size_t)r * dim;
  const int nchunks = dim >> 3;
  float acc = 0.0f;
  for (int c = lane; c < nchunks; c += 32) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c * 8);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = bf_lo(u[i]), hi = bf_hi(u[i]);
      acc = __fmaf_rn(lo, lo, acc);
      acc = __fmaf_rn(hi, hi, acc);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  const float rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)dim), eps)));
  for (int c = lane; c < nchunks; c += 32) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c * 8);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + c * 8);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    const uint32_t wu[4] = {wv.x, wv.y, wv.z, wv.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint16_t lo = f2bf(__fmul_rn(rbf(__fmul_rn(bf_lo(u[i]), rr)), bf_lo(wu[i])));
      const uint16_t hi = f2bf(__fmul_rn(rbf(__fmul_rn(bf_hi(u[i]), rr)), bf_hi(wu[i])));
      o[i] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint4*>(out + (size_t)r * dim + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// The Gemma4 block's combine (gemma4.rs:1079-1083): out[t] (f32) = sum over j in order of
// f32(y[t, j]) * w[t, j], the weights and the sum in f32 (its expert outputs and weights
// are f32 in the reference; y here is the bf16 output of the down projection).
__global__ void __launch_bounds__(256) combine_f32_kernel(CombineArgs a) {
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
  for (int j = 0; j < a.k; ++j) {
    const int64_t p = (int64_t)t * a.k + j;
    const float w = a.weights_f32[p];
    const uint4 v = *reinterpret_cast<const uint4*>(a.y + (size_t)a.inv[p] * a.H + h);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[2 * i] = __fadd_rn(acc[2 * i], __fmul_rn(bf_lo(u[i]), w));
      acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __fmul_rn(bf_hi(u[i]), w));
    }
  }
  float4* o = reinterpret_cast<float4*>(a.out_f32 + (size_t)t * a.H + h);
  o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
  o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

// out[r] = f32(bf16(x[r] * rsqrt(mean(x[r]^2) + eps))) * root * f32(scale): the Gemma4
// router's input (gemma4.rs:911-919: fast_rms_norm with a ones weight, then two multiplies
// by 0-d f32 arrays, which makes the rest of the router f32). The norm as rms_norm_kernel.
__global__ void __launch_bounds__(256) gemma_router_input_kernel(const uint16_t* __restrict__ x,
                                                                 const uint16_t* __restrict__ scale, float root,
                                                                 float eps, int64_t rows, int dim,
                                                                 float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  pdl_wait();
  pdl_trigger();
  if (r >= rows) return;
  const uint16_t* xr = x + (size_t)r * dim;
  const int nchunks = dim >> 3;
  float acc = 0.0f;
  for (int c = lane; c < nchunks; c += 32) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c * 8);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float lo = bf_lo(u[i]), hi = bf_hi(u[i]);
      acc = __fmaf_rn(lo, lo, acc);
      acc = __fmaf_rn(hi, hi, acc);
    }
  }
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
  const float rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, (float)dim), eps)));
  for (int c = lane; c < nchunks; c += 32) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + c * 8);
    const uint4 sv = *reinterpret_cast<const uint4*>(scale + c * 8);
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
    const uint32_t su[4] = {sv.x, sv.y, sv.z, sv.w};
    float o[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[2 * i] = __fmul_rn(__fmul_rn(rbf(__fmul_rn(bf_lo(u[i]), rr)), root), bf_lo(su[i]));
      o[2 * i + 1] = __fmul_rn(__fmul_rn(rbf(__fmul_rn(bf_hi(u[i]), rr)), root), bf_hi(su[i]));
    }
    float4* op = reinterpret_cast<float4*>(out + (size_t)r * dim + c * 8);
    op[0] = make_float4(o[0], o[1], o[2], o[3]);
    op[1] = make_float4(o[4], o[5], o[6], o[7]);
  }
}

cudaError_t launch_combine(const CombineArgs& a, cudaStream_t st) {
  const int64_t n = (int64_t)a.T * (a.H >> 3);
  if (n <= 0) return cudaSuccess;
  if (a.weights_f32) return launch_k(combine_f32_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, a);
  return launch_k(combine_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st, a);
}

cudaError_t launch_gemma_router_input(const uint16_t* x, const uint16_t* scale, float root, float eps, int64_t rows,
                                      int dim, float* out, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  return launch_k(gemma_router_input_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, st, x, scale, root, eps,
                  rows, dim, out);
}

cudaError_t launch_rms_norm(const uint16_t* x, const uint16_t* w, float eps, int64_t rows, int dim,
                            uint16_t* out, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  return launch_k(rms_norm_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, st, x, w, eps, rows, dim, out);
}

}  // namespace moe
