// norm.cu -- row-wise normalisations of a transformer block, over the last axis of a
// [rows, d] tensor stored as f32 or f16 (arithmetic in f32):
//   LayerNorm  y = gamma[i] * ((x - mean) / sqrt(var + eps)) + beta[i], mean and biased variance
//              over the row (lightship-core/src/operator/layernorm.rs:153-205)
//   Softmax    y = exp(x - max) * (1 / sum(exp(x - max))) (operator/softmax.rs:106-146)
// Rows of up to 1024 elements (d a multiple of 4, 16-byte aligned tensors) run one warp per
// row with the row held in registers: one read and one write of HBM per element.  Longer or
// unaligned rows run one CTA per row, re-reading the row on every pass (from L1/L2).  Either
// may update in place.  Reductions are tree-ordered, so results agree with the reference's
// sequential f32 sums within a rounding tolerance, not bit for bit.  LayerNorm can write its
// output quantized to int8 (per-tensor scale, the Quantize operator's rounding), which saves
// the f32 round trip when the next operator is an INT8 projection.
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

// CUDA's single-precision expf (within 2 ulp); the reference's f32::exp is the platform expf.
__device__ __forceinline__ float exp_f32(float v) { return expf(v); }

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
    for (int64_t i = threadIdx.x; i < d; i += kNormThreads) s = __fadd_rn(s, exp_f32(__fsub_rn(ld_val(xr, i), m)));
    s = block_sum(s, red);
    if (s > 0.0f) {
      const float scale = __fdiv_rn(1.0f, s);
      for (int64_t i = threadIdx.x; i < d; i += kNormThreads)
        st_val(yr, i, __fmul_rn(exp_f32(__fsub_rn(ld_val(xr, i), m)), scale));
    } else if (x != y) {
      for (int64_t i = threadIdx.x; i < d; i += kNormThreads) st_val(yr, i, ld_val(xr, i));
    }
  }
}

// ---------------------------------------------------------------- warp-per-row kernels
constexpr int kRowWarps = 8;  // rows per CTA

// four consecutive elements at p[i..i+3] (16-byte aligned for f32, 8-byte for f16)
__device__ __forceinline__ void ld4(const float* p, int64_t i, float (&v)[4]) {
  const float4 t = *reinterpret_cast<const float4*>(p + i);
  v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
}
__device__ __forceinline__ void ld4(const __half* p, int64_t i, float (&v)[4]) {
  const uint2 t = *reinterpret_cast<const uint2*>(p + i);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&t.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&t.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}
__device__ __forceinline__ void st4(float* p, int64_t i, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p + i) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void st4(__half* p, int64_t i, const float (&v)[4]) {
  const __half2 a = __floats2half2_rn(v[0], v[1]);
  const __half2 b = __floats2half2_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(p + i) = make_uint2(*reinterpret_cast<const uint32_t*>(&a),
                                               *reinterpret_cast<const uint32_t*>(&b));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Softmax over rows of d <= 128*J elements: lane l holds elements 128*j + 4*l .. +3.
template <typename T, int J>
__global__ void __launch_bounds__(kRowWarps * 32) softmax_rows_kernel(const T* x, T* y, int64_t rows, int d) {
  const int lane = threadIdx.x & 31;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5); r < rows;
       r += static_cast<int64_t>(gridDim.x) * kRowWarps) {
    const T* xr = x + r * d;
    float v[J][4];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int i = 128 * j + 4 * lane;
      if (i < d) {
        ld4(xr, i, v[j]);
      } else {
        v[j][0] = v[j][1] = v[j][2] = v[j][3] = -INFINITY;
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) m = fmaxf(m, v[j][e]);
    }
    m = warp_max(m);
    float s = 0.0f;
    float ex[J][4];
#pragma unroll
    for (int j = 0; j < J; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        ex[j][e] = exp_f32(__fsub_rn(v[j][e], m));
        if (128 * j + 4 * lane < d) s = __fadd_rn(s, ex[j][e]);
      }
    s = warp_sum(s);
    T* yr = y + r * d;
    if (s > 0.0f) {
      const float scale = __fdiv_rn(1.0f, s);
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int i = 128 * j + 4 * lane;
        if (i < d) {
          float o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) o[e] = __fmul_rn(ex[j][e], scale);
          st4(yr, i, o);
        }
      }
    } else if (x != y) {
#pragma unroll
      for (int j = 0; j < J; ++j) {
        const int i = 128 * j + 4 * lane;
        if (i < d) st4(yr, i, v[j]);
      }
    }
  }
}

// LayerNorm over rows of d <= 128*J elements, output T, or int8 when q != nullptr
// (q = R(y / s_out), saturated; the Quantize operator's arithmetic).
// a / b with y = RN(1 / b) computed once per row: q = RN(a y), r = a - q b (exact by FMA),
// RN(q + r y) -- Markstein's division by way of a correctly rounded reciprocal (P. Markstein,
// IBM J. Res. Dev. 34(1), 1990), which returns RN(a / b) while q stays in the normal range.
// Zero, tiny, huge and non-finite quotients take the IEEE division.
__device__ __forceinline__ float div_by_row(float a, float b, float y) {
  const float q = __fmul_rn(a, y);
  const float aq = fabsf(q);
  if (!(aq > 7.5e-37f && aq < 1.3e36f)) return __fdiv_rn(a, b);
  return __fmaf_rn(__fmaf_rn(-q, b, a), y, q);
}

template <typename T, int J, int RND>
__global__ void __launch_bounds__(kRowWarps * 32, 4) layernorm_rows_kernel(const T* x, T* y, int8_t* q, int64_t rows,
                                                                        int d, const float* __restrict__ gamma,
                                                                        const float* __restrict__ beta, float eps,
                                                                        float s_out, float inv_s, bool gb16) {
  const int lane = threadIdx.x & 31;
  const float fd = static_cast<float>(d);
  griddep_wait();  // launched as a dependent kernel: inputs and outputs are settled from here on
  griddep_launch_dependents();
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kRowWarps + (threadIdx.x >> 5); r < rows;
       r += static_cast<int64_t>(gridDim.x) * kRowWarps) {
    const T* xr = x + r * d;
    float v[J][4];
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int i = 128 * j + 4 * lane;
      if (i < d) {
        ld4(xr, i, v[j]);
#pragma unroll
        for (int e = 0; e < 4; ++e) s = __fadd_rn(s, v[j][e]);
      }
    }
    const float mean = __fdiv_rn(warp_sum(s), fd);
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < J; ++j) {
      if (128 * j + 4 * lane < d) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float t = __fsub_rn(v[j][e], mean);
          sq = __fadd_rn(sq, __fmul_rn(t, t));
        }
      }
    }
    const float var = __fdiv_rn(warp_sum(sq), fd);
    const float sd = __fsqrt_rn(__fadd_rn(var, eps));
    const float inv_sd = __frcp_rn(sd);
#pragma unroll
    for (int j = 0; j < J; ++j) {
      const int i = 128 * j + 4 * lane;
      if (i >= d) continue;
      float o[4];
      // gamma and beta as 16-byte vectors when they are 16-byte aligned (d is a multiple of 4)
      float gv[4] = {0.f, 0.f, 0.f, 0.f}, bv[4] = {0.f, 0.f, 0.f, 0.f};
      if (gb16) {
        if (gamma) {
          const float4 g4 = __ldg(reinterpret_cast<const float4*>(gamma + i));
          gv[0] = g4.x; gv[1] = g4.y; gv[2] = g4.z; gv[3] = g4.w;
        }
        if (beta) {
          const float4 b4 = __ldg(reinterpret_cast<const float4*>(beta + i));
          bv[0] = b4.x; bv[1] = b4.y; bv[2] = b4.z; bv[3] = b4.w;
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (gamma) gv[e] = __ldg(gamma + i + e);
          if (beta) bv[e] = __ldg(beta + i + e);
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float t = div_by_row(__fsub_rn(v[j][e], mean), sd, inv_sd);
        if (gamma) t = __fmul_rn(gv[e], t);
        if (beta) t = __fadd_rn(t, bv[e]);
        o[e] = t;
      }
      if (q) {
        // the four codes by the two-lane form of the same requantization (identical results)
        uint32_t pk[1];
        requant_pack_rnd<4, RND>(o, s_out, inv_s, false, pk);
        *reinterpret_cast<uint32_t*>(q + r * d + i) = pk[0];
      } else {
        st4(y + r * d, i, o);
      }
    }
  }
}

template <typename T, int RND>
lsc_status layernorm_rows(const T* x, T* y, int8_t* q, int64_t rows, int d, const float* gamma, const float* beta,
                          float eps, float s_out, float inv_s, int grid, bool overlap, cudaStream_t st) {
  const int j = (d + 127) / 128;
  const bool gb16 = ((reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(beta)) & 15) == 0;
#define LSC_LN_CASE(J)                                                                                          \
  case J:                                                                                                     \
    LSC_CUDA_TRY(launch_dependent(overlap, layernorm_rows_kernel<T, J, RND>, dim3(grid), dim3(kRowWarps * 32), 0, \
                                  st, x, y, q, rows, d, gamma, beta, eps, s_out, inv_s, gb16));                 \
    break;
  switch (j) {
    LSC_LN_CASE(1) LSC_LN_CASE(2) LSC_LN_CASE(3) LSC_LN_CASE(4) LSC_LN_CASE(5) LSC_LN_CASE(6) LSC_LN_CASE(7)
    LSC_LN_CASE(8)
    default: return set_error(LSC_ERROR_INVALID_ARGUMENT, "layernorm: row too long for the warp kernel");
  }
#undef LSC_LN_CASE
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

template <typename T>
lsc_status softmax_rows(const T* x, T* y, int64_t rows, int d, int grid, cudaStream_t st) {
  const int j = (d + 127) / 128;
#define LSC_SM_CASE(J)                                                                 \
  case J:                                                                            \
    softmax_rows_kernel<T, J><<<grid, kRowWarps * 32, 0, st>>>(x, y, rows, d);      \
    break;
  switch (j) {
    LSC_SM_CASE(1) LSC_SM_CASE(2) LSC_SM_CASE(3) LSC_SM_CASE(4) LSC_SM_CASE(5) LSC_SM_CASE(6) LSC_SM_CASE(7)
    LSC_SM_CASE(8)
    default: return set_error(LSC_ERROR_INVALID_ARGUMENT, "softmax: row too long for the warp kernel");
  }
#undef LSC_SM_CASE
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

// rows of d elements fit the warp kernels: d a multiple of 4 up to 1024, 16-byte aligned bases
bool rows_fit_warp(const void* x, const void* y, const void* q, int64_t d) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(q);
  return d > 0 && d <= 1024 && d % 4 == 0 && (a & 15) == 0;
}

int rows_grid(int64_t rows, int sm_count) {
  const int64_t ctas = (rows + kRowWarps - 1) / kRowWarps;
  const int64_t cap = static_cast<int64_t>(sm_count) * 16;
  return static_cast<int>(ctas < cap ? (ctas < 1 ? 1 : ctas) : cap);
}

int norm_grid(int64_t rows, int sm_count) {
  const int64_t cap = static_cast<int64_t>(sm_count) * 8;
  return static_cast<int>(rows < cap ? (rows < 1 ? 1 : rows) : cap);
}

}  // namespace

lsc_status launch_layernorm(const void* x, void* y, int32_t dtype, int64_t rows, int64_t d, const float* gamma,
                            const float* beta, float eps, cudaStream_t st, int8_t* q, float q_scale, int rounding) {
  if (rows < 0 || d < 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "layernorm: negative size");
  if (rows == 0 || d == 0) return LSC_SUCCESS;
  if (dtype != LSC_DTYPE_F32 && dtype != LSC_DTYPE_F16)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "layernorm: f32 or f16 tensors only");
  if (q && !(q_scale > 0.0f)) return set_error(LSC_ERROR_INVALID_ARGUMENT, "layernorm: int8 output needs a scale > 0");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const void* out = q ? static_cast<const void*>(q) : y;
  if (rows_fit_warp(x, out, nullptr, d)) {
    const int grid = rows_grid(rows, ds->sm_count);
    const float inv = q ? reciprocal_or_zero(q_scale) : 0.0f;
    const int di = static_cast<int>(d);
    const bool even = rounding == LSC_ROUND_HALF_EVEN;
    if (dtype == LSC_DTYPE_F32) {
      const float* xs = static_cast<const float*>(x);
      float* ys = static_cast<float*>(y);
      return even ? layernorm_rows<float, LSC_ROUND_HALF_EVEN>(xs, ys, q, rows, di, gamma, beta, eps, q_scale, inv, grid, ds->overlap_launches, st)
                  : layernorm_rows<float, LSC_ROUND_HALF_AWAY>(xs, ys, q, rows, di, gamma, beta, eps, q_scale, inv, grid, ds->overlap_launches, st);
    }
    const __half* xh = static_cast<const __half*>(x);
    __half* yh = static_cast<__half*>(y);
    return even ? layernorm_rows<__half, LSC_ROUND_HALF_EVEN>(xh, yh, q, rows, di, gamma, beta, eps, q_scale, inv, grid, ds->overlap_launches, st)
                : layernorm_rows<__half, LSC_ROUND_HALF_AWAY>(xh, yh, q, rows, di, gamma, beta, eps, q_scale, inv, grid, ds->overlap_launches, st);
  }
  if (q)
    return set_error(LSC_ERROR_UNSUPPORTED_LAYOUT,
                     "layernorm: an int8 output needs rows of at most 1024 elements, a multiple of 4, 16-byte aligned");
  const int grid = norm_grid(rows, ds->sm_count);
  if (dtype == LSC_DTYPE_F32)
    layernorm_kernel<float><<<grid, kNormThreads, 0, st>>>(static_cast<const float*>(x), static_cast<float*>(y), rows,
                                                           d, gamma, beta, eps);
  else
    layernorm_kernel<__half><<<grid, kNormThreads, 0, st>>>(static_cast<const __half*>(x), static_cast<__half*>(y),
                                                            rows, d, gamma, beta, eps);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

lsc_status launch_softmax(const void* x, void* y, int32_t dtype, int64_t rows, int64_t d, cudaStream_t st) {
  if (rows < 0 || d < 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "softmax: negative size");
  if (rows == 0 || d == 0) return LSC_SUCCESS;
  if (dtype != LSC_DTYPE_F32 && dtype != LSC_DTYPE_F16)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "softmax: f32 or f16 tensors only");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (rows_fit_warp(x, y, nullptr, d)) {
    const int grid = rows_grid(rows, ds->sm_count);
    if (dtype == LSC_DTYPE_F32)
      return softmax_rows(static_cast<const float*>(x), static_cast<float*>(y), rows, static_cast<int>(d), grid, st);
    return softmax_rows(static_cast<const __half*>(x), static_cast<__half*>(y), rows, static_cast<int>(d), grid, st);
  }
  const int grid = norm_grid(rows, ds->sm_count);
  if (dtype == LSC_DTYPE_F32)
    softmax_kernel<float><<<grid, kNormThreads, 0, st>>>(static_cast<const float*>(x), static_cast<float*>(y), rows, d);
  else
    softmax_kernel<__half><<<grid, kNormThreads, 0, st>>>(static_cast<const __half*>(x), static_cast<__half*>(y),
                                                          rows, d);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

}  // namespace lsc
