// common.cuh — device helpers shared by the MoE kernels (sm_100a).
//
// Numerics contract: every bf16 result is produced by rounding an fp32 value to
// nearest-even (f2bf), after each operation of the reference's bf16 graph. Every
// floating-point operation whose bits must match the CPU oracle is written with an
// explicit __f*_rn intrinsic so nvcc cannot contract or reorder it.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define MOE_DEV __device__ __forceinline__

namespace moe {

MOE_DEV float bf2f(uint16_t h) { return __uint_as_float(((uint32_t)h) << 16); }

// Round-to-nearest-even fp32 -> bf16 bits (NaN kept quiet).
MOE_DEV uint16_t f2bf(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

MOE_DEV float rbf(float f) { return bf2f(f2bf(f)); }

// bf16 pair packed in a uint32 (low half = first element).
MOE_DEV float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
MOE_DEV float bf_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// exp(x): Cody-Waite range reduction (W. J. Cody, W. Waite, "Software Manual for the
// Elementary Functions", 1980) with ln2 split into a 12-bit-short high part and a low
// part, then the degree-7 Taylor polynomial of exp(r) (coefficients 1/i!) in Horner
// form, scaled by 2^n. x > 88 gives +inf and x < -87 gives 0 by definition. The
// operation sequence is the one the CPU oracle evaluates, so both give the same bits.
MOE_DEV float exp_canon(float x) {
  if (x != x) return x;
  if (x > 88.0f) return __int_as_float(0x7f800000);
  if (x < -87.0f) return 0.0f;
  const float t = __fmul_rn(x, 0x1.715476p+0f);
  const float n = rintf(t);
  float r = __fmaf_rn(-n, 0x1.62ep-1f, x);
  r = __fmaf_rn(-n, 0x1.0bfbe8p-15f, r);
  float p = 0x1.a01a02p-13f;
  p = __fmaf_rn(p, r, 0x1.6c16c2p-10f);
  p = __fmaf_rn(p, r, 0x1.111112p-7f);
  p = __fmaf_rn(p, r, 0x1.555556p-5f);
  p = __fmaf_rn(p, r, 0x1.555556p-3f);
  p = __fmaf_rn(p, r, 0x1.0p-1f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = (int)n;
  const float scale = __uint_as_float((uint32_t)(ni + 127) << 23);
  return __fmul_rn(p, scale);
}

// sigmoid(x) = 1 / (1 + exp(-x)) with IEEE add and divide.
MOE_DEV float sigmoid_canon(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_canon(-x))); }

// h = bf16(bf16(g * bf16(sigmoid(g))) * u): the reference's
// x_gate.multiply(x_gate.sigmoid()).multiply(x_up) with bf16 results per op.
MOE_DEV uint16_t swiglu_bf16(float g, float u) {
  const float sg = rbf(sigmoid_canon(g));
  const float a = rbf(__fmul_rn(g, sg));
  return f2bf(__fmul_rn(a, u));
}

// h = bf16(gelu_approx(g) * u) for the Gemma4 SwitchGLU (gemma4.rs:308-322, 1049): the
// reference evaluates in f32 (its constants are 0-d f32 arrays):
//   0.5 * (g * (1 + tanh(sqrt(2/pi) * (g + 0.044715 * g^3)))) * u,
// with g^3 as two multiplies (the reference's power(x, 3)) and CUDA's tanhf; the product is
// rounded to bf16, the operand type of the down projection's MMA (the reference keeps f32).
MOE_DEV uint16_t gelu_mul_bf16(float g, float u) {
  const float x3 = __fmul_rn(__fmul_rn(g, g), g);
  const float inner = __fmul_rn(__fadd_rn(g, __fmul_rn(x3, 0x1.6e4e26p-5f)), 0x1.988452p-1f);
  const float gate = __fadd_rn(1.0f, tanhf(inner));
  const float h = __fmul_rn(0.5f, __fmul_rn(g, gate));
  return f2bf(__fmul_rn(h, u));
}

// Programmatic dependent launch: kernels of the block are launched so that each may
// start while its predecessor in the stream drains. pdl_wait() blocks until the
// predecessor grid has completed and its writes are visible (a no-op when the kernel
// was launched normally); it must precede every read of a predecessor's output.
// pdl_trigger() lets the next kernel start launching once every CTA has called it.
MOE_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
MOE_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

}  // namespace moe
