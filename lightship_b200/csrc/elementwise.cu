// elementwise.cu -- FP32 per-element operators of the dense path that stand alone when no
// contraction precedes them:
//   BatchNorm inference  y = gamma * ((x - mean) * inv_std) + beta, inv_std = 1/sqrt(var + eps)
//                        (lightship-core/src/operator/batchnorm.rs:154-215; inv_std is computed
//                        on the host with the same f32 operations), optional ReLU
//                        (FusionType::BatchNormReLU, backend/cpu.rs:404-439)
//   ReLU / ReLU6 / SiLU / GELU (platform/simd.rs:552-562, operator/silu.rs:47-61,
//                        operator/gelu.rs:77-103)
//   Add (+ReLU)          (backend/cpu.rs:468-517; FusionType::AddReLU)
// Every operation is an explicitly rounded intrinsic, so results match the reference bit
// for bit.  16-byte vector loads where alignment allows; grids are a multiple of the SM count.
#include "epilogue.cuh"
#include "lsc_internal.h"

namespace lsc {
namespace {

__device__ __forceinline__ float act_any(float x, int act) {
  switch (act) {
    case LSC_ACT_RELU: return act_relu(x);
    case LSC_ACT_RELU6: return act_relu6(x);
    case LSC_ACT_SILU: return act_silu(x);
    case LSC_ACT_GELU: return act_gelu(x);
    default: return x;
  }
}

__global__ void batchnorm_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t total,
                                 int64_t channels, int64_t spatial, const float* __restrict__ gamma,
                                 const float* __restrict__ beta, const float* __restrict__ mean,
                                 const float* __restrict__ inv_std, int act) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t c = (i / spatial) % channels;
    const float xn = __fmul_rn(__fsub_rn(__ldg(x + i), __ldg(mean + c)), __ldg(inv_std + c));
    const float v = __fadd_rn(__fmul_rn(__ldg(gamma + c), xn), __ldg(beta + c));
    y[i] = act_any(v, act);
  }
}

__global__ void activation_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t n,
                                  int act) {
  const int64_t n4 = n / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const bool vec = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  int64_t start = 0;
  if (vec) {
    for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < n4; v += stride) {
      float4 f = __ldg(reinterpret_cast<const float4*>(x) + v);
      f.x = act_any(f.x, act);
      f.y = act_any(f.y, act);
      f.z = act_any(f.z, act);
      f.w = act_any(f.w, act);
      reinterpret_cast<float4*>(y)[v] = f;
    }
    start = n4 * 4;
  }
  for (int64_t i = start + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    y[i] = act_any(__ldg(x + i), act);
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b,
                           float* __restrict__ y, int64_t n, int act) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[i] = act_any(__fadd_rn(__ldg(a + i), __ldg(b + i)), act);
}

int grid_ew(int64_t n, int sm_count) {
  int64_t g = (n + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count) * 8;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

lsc_status launch_batchnorm_f32(const float* x, float* y, int64_t n, int64_t c, int64_t spatial,
                                const float* gamma, const float* beta, const float* mean,
                                const float* inv_std, int act, cudaStream_t st) {
  const int64_t total = n * c * spatial;
  if (total == 0) return LSC_SUCCESS;
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  batchnorm_kernel<<<grid_ew(total, ds->sm_count), 256, 0, st>>>(x, y, total, c, spatial, gamma,
                                                                  beta, mean, inv_std, act);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

lsc_status launch_activation_f32(const float* x, float* y, int64_t n, int act, cudaStream_t st) {
  if (n == 0) return LSC_SUCCESS;
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  activation_kernel<<<grid_ew((n + 3) / 4, ds->sm_count), 256, 0, st>>>(x, y, n, act);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

lsc_status launch_add_f32(const float* a, const float* b, float* y, int64_t n, int act,
                          cudaStream_t st) {
  if (n == 0) return LSC_SUCCESS;
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  add_kernel<<<grid_ew(n, ds->sm_count), 256, 0, st>>>(a, b, y, n, act);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

}  // namespace lsc
