// epilogue.cuh -- the INT8 chain's per-element epilogue, written to give the same bits as
// LightShip's CPU math:
//   acc += bias[n]                         (i32, wrapping)
//   y    = (f32)acc * scale[n]             dequantize   core/cpu/quantized_ops.rs:36-40
//   y    = act(y)                          ReLU         core/platform/simd.rs:552-556
//                                          ReLU6        core/platform/simd.rs:558-562
//                                          SiLU         core/operator/silu.rs:47-61
//   q    = (i8)clamp(R(y / s_out), -128, 127)           core/cpu/quantized_ops.rs:43-48
// Every operation is an explicitly rounded intrinsic so nvcc cannot contract it into an
// FMA or replace the IEEE division.
#pragma once
#include <stdint.h>

#include "lightship_cuda.h"

namespace lsc {

__device__ __forceinline__ float act_relu(float x) { return x > 0.0f ? x : 0.0f; }

// Rust f32::clamp(0, 6): NaN (with its payload) and -0.0 pass through unchanged.  The NaN
// test comes first so the compiler cannot lower the clamp to min/max instructions, which
// return the canonical NaN.
__device__ __forceinline__ float act_relu6(float x) {
  if (x != x) return x;
  float r = x;
  if (r < 0.0f) r = 0.0f;
  if (r > 6.0f) r = 6.0f;
  return r;
}

// x / (1 + exp(-x)) with the reference's +-20 cut-offs.  exp is evaluated in double and
// rounded once to f32, which gives the correctly rounded expf for all but a vanishing set
// of inputs; the reference's expf is glibc's (error < 0.502 ulp).  The two are compared
// over the whole [-20, 20] float range by the tests.
__device__ __forceinline__ float act_silu(float x) {
  if (x > 20.0f) return x;
  if (x < -20.0f) return 0.0f;
  const float e = __double2float_rn(exp(-static_cast<double>(x)));
  return __fdiv_rn(x, __fadd_rn(1.0f, e));
}

template <int ACT>
__device__ __forceinline__ float apply_act(float x) {
  if constexpr (ACT == LSC_ACT_RELU) return act_relu(x);
  else if constexpr (ACT == LSC_ACT_RELU6) return act_relu6(x);
  else if constexpr (ACT == LSC_ACT_SILU) return act_silu(x);
  else return x;
}

// R(t) then Rust's clamp(-128,127) `as i8`: NaN -> 0.
template <int RND>
__device__ __forceinline__ int32_t requant_i8(float y, float s_out) {
  const float t = __fdiv_rn(y, s_out);
  float r = (RND == LSC_ROUND_HALF_EVEN) ? rintf(t) : roundf(t);
  if (r != r) return 0;
  if (r < -128.0f) r = -128.0f;
  if (r > 127.0f) r = 127.0f;
  return __float2int_rz(r);
}

__device__ __forceinline__ float dequant(int32_t acc, float scale) {
  return __fmul_rn(__int2float_rn(acc), scale);
}

}  // namespace lsc
