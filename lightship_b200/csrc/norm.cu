// norm.cu -- row-wise normalisations of a transformer block, over the last axis of a
// [rows, d] tensor stored as f32 or f16 (arithmetic in f32):
//   LayerNorm  y = gamma[i] * ((x - mean) / sqrt(var + eps)) + beta[i], mean and biased variance
//              over the row (lightship-core/src/operator/layernorm.rs:153-205)
//   Softmax    y = exp(x - max) * (1 / sum(exp(x - max))) (operator/softmax.rs:106-146)
// One CTA per row (grid-stride over rows); the row is read from global memory on every pass
// (it stays in L1/L2 between passes) and may be updated in place.  Reductions are
// tree-ordered, so results agree with the reference's sequential f32 sums within a rounding
// tolerance, not bit for bit.
#include <cuda_fp16.h>

#include "epilogue.cuh"
#include "lsc_internal.h"

namespace lsc {
namespace {

constexpr int kNormThreads = 256;

template <typename T>
__device__ __forceinline__ float ld_val(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld_val<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld_val<__half>(const __half* p, int64_t i) { return __half2float(p[i]); }

__device__ __forceinline__ void st_val(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void st_val(__half* p, int64_t i, float v) { p[i] = __float2half_rn(v); }

// Sum over the CTA; every thread gets the total.
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = 0.0f;
  if (lane < kNormThreads / 32) t = red[lane];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
  return t;
}

// Max over the CTA (f32::max semantics: NaN operands are ignored).
__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  float t = -INFINITY;
  if (lane < kNormThreads / 32) t = red[lane];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
  return t;
}

template <typename T>
__global__ void __launch_bounds__(kNormThreads) layernorm_kernel(const T* x, T* y,
                                                                 int64_t rows, int64_t d,
                                                                 const float* __restrict__ gamma,
                                                                 const float* __restrict__ beta, float eps) {
  __shared__ float red[kNormThreads / 32];
  const float fd = static_cast<float>(d);
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * d;
    T* yr = y + r * d;
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < d; i += kNormThreads) s = __fadd_rn(s, ld_val(xr, i));
    const float mean = __fdiv_rn(block_sum(s, red), fd);
    float q = 0.0f;
    for (int64_t i = threadIdx.x; i < d; i += kNormThreads) {
      const float t = __fsub_rn(ld_val(xr, i), mean);
      q = __fadd_rn(q, __fmul_rn(t, t));
    }
    const float var = __fdiv_rn(block_sum(q, red), fd);
    const float sd = __fsqrt_rn(__fadd_rn(var, eps));
    for (int64_t i = threadIdx.x; i < d; i += kNormThreads) {
      float v = __fdiv_rn(__fsub_rn(ld_val(xr, i), mean), sd);
      if (gamma) v = __fmul_rn(__ldg(gamma + i), v);
      if (beta) v = __fadd_rn(v, __ldg(beta + i));
      st_val(yr, i, v);
    }
  }
}

// exp rounded once from double: the correctly rounded expf for all but a vanishing set of
// inputs (the reference's f32::exp is the platform expf).
__device__ __forceinline__ float exp_rn(float v) { return __double2float_rn(exp(static_cast<double>(v))); }

template <typename T>
__global__ void __launch_bounds__(kNormThreads) softmax_kernel(const T* x, T* y,
                                                               int64_t rows, int64_t d) {
  __shared__ float red[kNormThreads / 32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const T* xr = x + r * d;
    T* yr = y + r * d;
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < d; i += kNormThreads) m = fmaxf(m, ld_val(xr, i));
    m = block_max(m, red);
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < d; i += kNormThreads) s = __fadd_rn(s, exp_rn(__fsub_rn(ld_val(xr, i), m)));
    s = block_sum(s, red);
    if (s > 0.0f) {
      const float scale = __fdiv_rn(1.0f, s);
      for (int64_t i = threadIdx.x; i < d; i += kNormThreads)
        st_val(yr, i, __fmul_rn(exp_rn(__fsub_rn(ld_val(xr, i), m)), scale));
    } else if (x != y) {
      for (int64_t i = threadIdx.x; i < d; i += kNormThreads) st_val(yr, i, ld_val(xr, i));
    }
  }
}

int norm_grid(int64_t rows, int sm_count) {
  const int64_t cap = static_cast<int64_t>(sm_count) * 8;
  return static_cast<int>(rows < cap ? (rows < 1 ? 1 : rows) : cap);
}

}  // namespace

lsc_status launch_layernorm(const void* x, void* y, int32_t dtype, int64_t rows, int64_t d, const float* gamma,
                            const float* beta, float eps, cudaStream_t st) {
  if (rows < 0 || d < 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "layernorm: negative size");
  if (rows == 0 || d == 0) return LSC_SUCCESS;
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const int grid = norm_grid(rows, ds->sm_count);
  if (dtype == LSC_DTYPE_F32)
    layernorm_kernel<float><<<grid, kNormThreads, 0, st>>>(static_cast<const float*>(x), static_cast<float*>(y), rows,
                                                           d, gamma, beta, eps);
  else if (dtype == LSC_DTYPE_F16)
    layernorm_kernel<__half><<<grid, kNormThreads, 0, st>>>(static_cast<const __half*>(x), static_cast<__half*>(y),
                                                            rows, d, gamma, beta, eps);
  else
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "layernorm: f32 or f16 tensors only");
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

lsc_status launch_softmax(const void* x, void* y, int32_t dtype, int64_t rows, int64_t d, cudaStream_t st) {
  if (rows < 0 || d < 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "softmax: negative size");
  if (rows == 0 || d == 0) return LSC_SUCCESS;
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const int grid = norm_grid(rows, ds->sm_count);
  if (dtype == LSC_DTYPE_F32)
    softmax_kernel<float><<<grid, kNormThreads, 0, st>>>(static_cast<const float*>(x), static_cast<float*>(y), rows, d);
  else if (dtype == LSC_DTYPE_F16)
    softmax_kernel<__half><<<grid, kNormThreads, 0, st>>>(static_cast<const __half*>(x), static_cast<__half*>(y),
                                                          rows, d);
  else
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "softmax: f32 or f16 tensors only");
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

}  // namespace lsc
