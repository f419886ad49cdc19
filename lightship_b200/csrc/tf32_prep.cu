// tf32_prep.cu -- operand preparation for the FP32 contractions on the tensor cores.
//
// The FP32 path (MatMul / FullyConnected / Conv2d, lightship-core/src/backend/cpu.rs:949-1290
// and core/operator/convolution.rs:90-267) runs as split-TF32: every f32 operand x is
// written as hi + lo with hi = x truncated to TF32 (low 13 mantissa bits cleared, exactly
// representable) and lo = x - hi (exact in f32).  The tensor cores then form
// hi*hi + hi*lo + lo*hi in f32, which recovers close to f32 accuracy.  These kernels write
// hi/lo in the layout the contraction kernel loads by TMA (K-major rows, NHWC for
// convolution inputs), transposing or re-laying out on the way.  All are HBM-bound.
#include "lsc_internal.h"

namespace lsc {
namespace {

__device__ __forceinline__ void split(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = __fsub_rn(x, hi);
}

// Row-major [rows, cols] -> hi/lo with the same layout (cols padded to ld with zeros).
__global__ void split_rows_kernel(const float* __restrict__ x, int64_t rows, int64_t cols,
                                  int64_t ld, float* __restrict__ hi, float* __restrict__ lo) {
  griddep_wait();  // launched as a dependent kernel: inputs and outputs are settled from here on
  griddep_launch_dependents();
  const int64_t total = rows * ld;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / ld, c = i - r * ld;
    float h = 0.0f, l = 0.0f;
    if (c < cols) split(__ldg(x + r * cols + c), h, l);
    hi[i] = h;
    if (lo) lo[i] = l;
  }
}

// [K, N] row-major -> transposed hi/lo [N, ldk] (K padded to ldk), through a shared tile.
__global__ void split_transpose_kernel(const float* __restrict__ x, int64_t k, int64_t n,
                                       int64_t ldk, float* __restrict__ hi,
                                       float* __restrict__ lo) {
  __shared__ float tile[32][33];
  griddep_wait();  // launched as a dependent kernel: inputs and outputs are settled from here on
  griddep_launch_dependents();
  const int64_t k0 = static_cast<int64_t>(blockIdx.y) * 32, n0 = static_cast<int64_t>(blockIdx.x) * 32;
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int64_t kk = k0 + j, nn = n0 + threadIdx.x;
    tile[j][threadIdx.x] = (kk < k && nn < n) ? __ldg(x + kk * n + nn) : 0.0f;
  }
  __syncthreads();
  for (int j = threadIdx.y; j < 32; j += blockDim.y) {
    const int64_t nn = n0 + j, kk = k0 + threadIdx.x;
    if (nn < n && kk < ldk) {
      float h, l;
      split(tile[threadIdx.x][j], h, l);
      hi[nn * ldk + kk] = h;
      if (lo) lo[nn * ldk + kk] = l;
    }
  }
}

// NCHW [N, C, H, W] -> NHWC hi/lo [N, H, W, Cp] (channels padded to Cp with zeros).
__global__ void split_nchw_to_nhwc_kernel(const float* __restrict__ x, int64_t n, int64_t c,
                                          int64_t hw, int64_t cp, float* __restrict__ hi,
                                          float* __restrict__ lo) {
  // one block per (image, 32-pixel strip); threads walk channels
  __shared__ float tile[32][33];
  griddep_wait();  // launched as a dependent kernel: inputs and outputs are settled from here on
  griddep_launch_dependents();
  const int64_t img = blockIdx.y;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * 32;
  for (int64_t c0 = 0; c0 < cp; c0 += 32) {
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
      const int64_t cc = c0 + j, pp = p0 + threadIdx.x;
      tile[j][threadIdx.x] = (cc < c && pp < hw) ? __ldg(x + (img * c + cc) * hw + pp) : 0.0f;
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
      const int64_t pp = p0 + j, cc = c0 + threadIdx.x;
      if (pp < hw && cc < cp) {
        float h, l;
        split(tile[threadIdx.x][j], h, l);
        const int64_t o = (img * hw + pp) * cp + cc;
        hi[o] = h;
        if (lo) lo[o] = l;
      }
    }
    __syncthreads();
  }
}

int grid_1d(int64_t n, int sm_count) {
  int64_t g = (n + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count) * 8;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

lsc_status prep_split_rows(const float* x, int64_t rows, int64_t cols, int64_t ld, float* hi,
                           float* lo, cudaStream_t st) {
  if (rows * ld == 0) return LSC_SUCCESS;
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, split_rows_kernel, dim3(grid_1d(rows * ld, ds->sm_count)),
                                dim3(256), 0, st, x, rows, cols, ld, hi, lo));
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

lsc_status prep_split_transpose(const float* x, int64_t k, int64_t n, int64_t ldk, float* hi,
                                float* lo, cudaStream_t st) {
  if (k == 0 || n == 0) return LSC_SUCCESS;
  if ((ldk + 31) / 32 > 65535) return set_error(LSC_ERROR_INVALID_ARGUMENT, "transpose: K too large");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const dim3 grid(static_cast<unsigned>((n + 31) / 32), static_cast<unsigned>((ldk + 31) / 32));
  LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, split_transpose_kernel, grid, dim3(32, 8), 0, st, x, k, n, ldk,
                                hi, lo));
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

lsc_status prep_split_nchw_to_nhwc(const float* x, int64_t n, int64_t c, int64_t hw, int64_t cp,
                                   float* hi, float* lo, cudaStream_t st) {
  if (n == 0 || hw == 0) return LSC_SUCCESS;
  if (n > 65535) return set_error(LSC_ERROR_INVALID_ARGUMENT, "nchw->nhwc: batch too large");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const dim3 grid(static_cast<unsigned>((hw + 31) / 32), static_cast<unsigned>(n));
  LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, split_nchw_to_nhwc_kernel, grid, dim3(32, 8), 0, st, x, n, c,
                                hw, cp, hi, lo));
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

}  // namespace lsc
