// quant.cu -- bandwidth kernels of the quantization operators:
//   quantize   q = clamp(sat_i32(R(v / s)) + zp, qmin, qmax)   quantization/helpers.rs:139-155
//   dequantize x = ((f32)q - (f32)zp) * s                       quantization/helpers.rs:158-160
//   find_scale_zp (min/max calibration)                         quantization/helpers.rs:101-136
// Per-tensor (quantize_tensor / dequantize_tensor, helpers.rs:11-94) and per-channel
// (QuantizationParameters per-channel, quantization/scheme.rs:58-121) forms.
// Loads and stores are 16-byte vectors; grids are a multiple of the SM count.
#include <mutex>

#include "lsc_internal.h"
#include "sm100.cuh"

namespace lsc {
namespace {

struct QRange {
  int32_t lo, hi;
};

// Clamp range of quantize_value / find_scale_zp (helpers.rs:109-114, :140-151): only the
// quantized types have their own range; every other dtype, plain I8 and I32 included, takes
// the `_` arm (0, 255).  The storage type is separate: I8 / QINT8 store int8 (a code above
// 127 wraps as Rust's `as i8`), I32 / QINT32 int32, U8 / QUINT8 uint8.
__host__ __device__ inline QRange qrange(int qdtype) {
  switch (qdtype) {
    case LSC_DTYPE_QINT8: return {-128, 127};
    case LSC_DTYPE_QINT32: return {INT32_MIN, INT32_MAX};
    default: return {0, 255};  // QUInt8 and the reference's `_` arm
  }
}

// Rust `f32 as i32`: saturating, NaN -> 0.
__device__ __forceinline__ int32_t sat_f32_i32(float v) {
  if (v != v) return 0;
  if (v >= 2147483648.0f) return INT32_MAX;
  if (v <= -2147483648.0f) return INT32_MIN;
  return __float2int_rz(v);
}

template <int RND>
__device__ __forceinline__ int32_t quantize_one(float v, float scale, int32_t zp, QRange r) {
  const float t = __fdiv_rn(v, scale);
  const float rr = RND == LSC_ROUND_HALF_EVEN ? rintf(t) : roundf(t);
  const int32_t q = static_cast<int32_t>(static_cast<uint32_t>(sat_f32_i32(rr)) +
                                         static_cast<uint32_t>(zp));  // wrapping i32 add
  return q < r.lo ? r.lo : (q > r.hi ? r.hi : q);
}

template <typename QT>
__device__ __forceinline__ void store_q(QT* out, int64_t i, int32_t q) {
  out[i] = static_cast<QT>(q);
}

// Per-tensor or per-channel (channel = (i / inner) % channels) quantization, 4 elements
// per thread per step, 16-byte loads.
template <typename QT, int RND>
__global__ void quantize_kernel(const float* __restrict__ x, QT* __restrict__ out, int64_t n,
                                const float* __restrict__ scales, const int32_t* __restrict__ zps,
                                float scale0, int32_t zp0, int32_t channels, int64_t inner,
                                int qdtype) {
  const QRange r = qrange(qdtype);
  const int64_t n4 = n / 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  for (int64_t v = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < n4;
       v += stride) {
    const int64_t i = v * 4;
    float e[4];
    if (vec) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(x) + v);
      e[0] = f.x; e[1] = f.y; e[2] = f.z; e[3] = f.w;
    } else {
#pragma unroll
      for (int t = 0; t < 4; ++t) e[t] = __ldg(x + i + t);
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float s = scale0;
      int32_t z = zp0;
      if (scales) {
        const int64_t c = ((i + t) / inner) % channels;
        s = __ldg(scales + c);
        z = zps ? __ldg(zps + c) : 0;
      }
      store_q(out, i + t, quantize_one<RND>(e[t], s, z, r));
    }
  }
  // tail
  for (int64_t i = n4 * 4 + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    float s = scale0;
    int32_t z = zp0;
    if (scales) {
      const int64_t c = (i / inner) % channels;
      s = __ldg(scales + c);
      z = zps ? __ldg(zps + c) : 0;
    }
    store_q(out, i, quantize_one<RND>(__ldg(x + i), s, z, r));
  }
}

template <typename QT>
__global__ void dequantize_kernel(const QT* __restrict__ q, float* __restrict__ out, int64_t n,
                                  const float* __restrict__ scales, const int32_t* __restrict__ zps,
                                  float scale0, int32_t zp0, int32_t channels, int64_t inner) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    float s = scale0;
    int32_t z = zp0;
    if (scales) {
      const int64_t c = (i / inner) % channels;
      s = __ldg(scales + c);
      z = zps ? __ldg(zps + c) : 0;
    }
    const int32_t v = static_cast<int32_t>(q[i]);
    out[i] = __fmul_rn(__fsub_rn(__int2float_rn(v), __int2float_rn(z)), s);
  }
}

// Order-preserving map of a float onto uint32 (for atomicMin/atomicMax).
__device__ __forceinline__ uint32_t fkey(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float fkey_inv(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// The reference's scale / zero point from the folded min/max keys.  No key (all inputs NaN
// or none) leaves the fold at (+inf, -inf), as the reference's fold does.
__device__ __forceinline__ void finalize_scale_zp(uint32_t gmin, uint32_t gmax, int qdtype,
                                                  int symmetric, float* scale_out,
                                                  int32_t* zp_out) {
  const float mn = gmin == 0xFFFFFFFFu ? __int_as_float(0x7f800000) : fkey_inv(gmin);
  const float mx = gmax == 0u ? -__int_as_float(0x7f800000) : fkey_inv(gmax);
  const QRange r = qrange(qdtype);
  if (symmetric) {
    const float am = fmaxf(fabsf(mx), fabsf(mn));
    *scale_out = am > 0.0f ? __fdiv_rn(am, static_cast<float>(r.hi)) : 1.0f;
    *zp_out = 0;
  } else {
    // (qmax - qmin) is an i32 subtraction in the reference; it wraps for QInt32.
    const int32_t span = static_cast<int32_t>(static_cast<uint32_t>(r.hi) - static_cast<uint32_t>(r.lo));
    const float s = mx > mn ? __fdiv_rn(__fsub_rn(mx, mn), static_cast<float>(span)) : 1.0f;
    const float z = __fsub_rn(static_cast<float>(r.lo), __fdiv_rn(mn, s));
    *scale_out = s;
    *zp_out = sat_f32_i32(roundf(z));
  }
}

// find_scale_zp: f32::min / f32::max fold (NaN skipped), then the reference's symmetric /
// asymmetric formulas, computed by the last block to finish.  ws = 3 x u32:
// [min key, max key, finished-block count]; it must be zeroed/initialised before launch.
__global__ void find_scale_zp_kernel(const float* __restrict__ x, int64_t n, int qdtype,
                                     int symmetric, uint32_t* ws, float* scale_out,
                                     int32_t* zp_out) {
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
  bool any = false;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    const float v = __ldg(x + i);
    if (v != v) continue;
    const uint32_t k = fkey(v);
    kmin = k < kmin ? k : kmin;
    kmax = k > kmax ? k : kmax;
    any = true;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t a = __shfl_xor_sync(0xFFFFFFFFu, kmin, o);
    const uint32_t b = __shfl_xor_sync(0xFFFFFFFFu, kmax, o);
    kmin = a < kmin ? a : kmin;
    kmax = b > kmax ? b : kmax;
  }
  any = __any_sync(0xFFFFFFFFu, any);
  if ((threadIdx.x & 31) == 0 && any) {
    atomicMin(&ws[0], kmin);
    atomicMax(&ws[1], kmax);
  }
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(&ws[2], 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  finalize_scale_zp(atomicAdd(&ws[0], 0u), atomicAdd(&ws[1], 0u), qdtype, symmetric, scale_out,
                    zp_out);
}

__global__ void init_minmax_ws(uint32_t* ws) {
  ws[0] = 0xFFFFFFFFu;
  ws[1] = 0u;
  ws[2] = 0u;
}

// Per-channel find_scale_zp over the rows of x [rows, cols] (channel = row, as for a
// weight [Cout, K]).  Block b handles chunk (b % chunks) of row (b / chunks); per-row
// partial keys and a finished-chunk count live in ws[3*row .. 3*row+2], and the last chunk
// of a row writes that row's scale and zero point.
__global__ void find_scale_zp_rows_kernel(const float* __restrict__ x, int64_t rows, int64_t cols,
                                          int64_t chunk, int32_t chunks, int qdtype,
                                          int symmetric, uint32_t* ws, float* scales,
                                          int32_t* zps) {
  const int64_t row = blockIdx.x / chunks;
  const int64_t part = blockIdx.x - row * chunks;
  if (row >= rows) return;
  const float* xr = x + row * cols;
  const int64_t begin = part * chunk;
  const int64_t end = begin + chunk < cols ? begin + chunk : cols;
  uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
  for (int64_t i = begin + threadIdx.x; i < end; i += blockDim.x) {
    const float v = __ldg(xr + i);
    if (v != v) continue;
    const uint32_t k = fkey(v);
    kmin = k < kmin ? k : kmin;
    kmax = k > kmax ? k : kmax;
  }
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t a = __shfl_xor_sync(0xFFFFFFFFu, kmin, o);
    const uint32_t b = __shfl_xor_sync(0xFFFFFFFFu, kmax, o);
    kmin = a < kmin ? a : kmin;
    kmax = b > kmax ? b : kmax;
  }
  uint32_t* w = ws + 3 * row;
  if ((threadIdx.x & 31) == 0) {
    if (kmin != 0xFFFFFFFFu) atomicMin(&w[0], kmin);
    if (kmax != 0u) atomicMax(&w[1], kmax);
  }
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) {
    __threadfence();
    last = atomicAdd(&w[2], 1u) == static_cast<uint32_t>(chunks - 1);
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  finalize_scale_zp(atomicAdd(&w[0], 0u), atomicAdd(&w[1], 0u), qdtype, symmetric, scales + row,
                    zps + row);
}

__global__ void init_minmax_rows(uint32_t* ws, int64_t rows) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < rows;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    ws[3 * i] = 0xFFFFFFFFu;
    ws[3 * i + 1] = 0u;
    ws[3 * i + 2] = 0u;
  }
}

int grid_for(int64_t work_items, int sm_count, int block) {
  const int64_t want = (work_items + block - 1) / block;
  const int64_t cap = static_cast<int64_t>(sm_count) * 8;
  const int64_t g = want < cap ? want : cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

bool valid_qdtype(int q) {
  return q == LSC_DTYPE_QINT8 || q == LSC_DTYPE_QUINT8 || q == LSC_DTYPE_QINT32 ||
         q == LSC_DTYPE_I8 || q == LSC_DTYPE_U8 || q == LSC_DTYPE_I32;
}

template <int RND>
lsc_status launch_quantize_r(const float* x, void* out, int64_t n, int qdtype,
                             const float* scales, const int32_t* zps, float scale0, int32_t zp0,
                             int32_t channels, int64_t inner, int grid, cudaStream_t st) {
  constexpr int B = 256;
  switch (qdtype) {
    case LSC_DTYPE_QINT8:
    case LSC_DTYPE_I8:
      quantize_kernel<int8_t, RND><<<grid, B, 0, st>>>(x, static_cast<int8_t*>(out), n, scales,
                                                       zps, scale0, zp0, channels, inner, qdtype);
      break;
    case LSC_DTYPE_QINT32:
    case LSC_DTYPE_I32:
      quantize_kernel<int32_t, RND><<<grid, B, 0, st>>>(x, static_cast<int32_t*>(out), n, scales,
                                                        zps, scale0, zp0, channels, inner, qdtype);
      break;
    default:
      quantize_kernel<uint8_t, RND><<<grid, B, 0, st>>>(x, static_cast<uint8_t*>(out), n, scales,
                                                        zps, scale0, zp0, channels, inner, qdtype);
  }
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

}  // namespace

lsc_status launch_quantize(const float* x, void* out, int64_t n, int qdtype, const float* scales,
                           const int32_t* zps, float scale0, int32_t zp0, int32_t channels,
                           int64_t inner, int rounding, cudaStream_t st) {
  if (n < 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantize: negative size");
  if (n == 0) return LSC_SUCCESS;
  if (!x || !out) return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantize: null pointer");
  if (!valid_qdtype(qdtype))
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "quantize: dtype %d is not a quantized type", qdtype);
  if (scales && (channels <= 0 || inner <= 0))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantize: bad channel layout");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const int grid = grid_for((n + 3) / 4, ds->sm_count, 256);
  if (rounding == LSC_ROUND_HALF_EVEN)
    return launch_quantize_r<LSC_ROUND_HALF_EVEN>(x, out, n, qdtype, scales, zps, scale0, zp0,
                                                  channels, inner, grid, st);
  return launch_quantize_r<LSC_ROUND_HALF_AWAY>(x, out, n, qdtype, scales, zps, scale0, zp0,
                                                channels, inner, grid, st);
}

lsc_status launch_dequantize(const void* q, int qdtype, float* out, int64_t n, const float* scales,
                             const int32_t* zps, float scale0, int32_t zp0, int32_t channels,
                             int64_t inner, cudaStream_t st) {
  if (n < 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "dequantize: negative size");
  if (n == 0) return LSC_SUCCESS;
  if (!q || !out) return set_error(LSC_ERROR_INVALID_ARGUMENT, "dequantize: null pointer");
  if (!valid_qdtype(qdtype))
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "dequantize: dtype %d is not a quantized type", qdtype);
  if (scales && (channels <= 0 || inner <= 0))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "dequantize: bad channel layout");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const int grid = grid_for(n, ds->sm_count, 256);
  switch (qdtype) {
    case LSC_DTYPE_QINT8:
    case LSC_DTYPE_I8:
      dequantize_kernel<int8_t><<<grid, 256, 0, st>>>(static_cast<const int8_t*>(q), out, n, scales,
                                                     zps, scale0, zp0, channels, inner);
      break;
    case LSC_DTYPE_QINT32:
    case LSC_DTYPE_I32:
      dequantize_kernel<int32_t><<<grid, 256, 0, st>>>(static_cast<const int32_t*>(q), out, n,
                                                      scales, zps, scale0, zp0, channels, inner);
      break;
    default:
      dequantize_kernel<uint8_t><<<grid, 256, 0, st>>>(static_cast<const uint8_t*>(q), out, n,
                                                      scales, zps, scale0, zp0, channels, inner);
  }
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

lsc_status launch_find_scale_zp(const float* x, int64_t n, int qdtype, int symmetric,
                                void* workspace, uint64_t workspace_bytes, float* scale_out,
                                int32_t* zp_out, cudaStream_t st) {
  if (n < 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "find_scale_zp: negative size");
  if (!scale_out || !zp_out)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "find_scale_zp: null output");
  if (n > 0 && !x) return set_error(LSC_ERROR_INVALID_ARGUMENT, "find_scale_zp: null input");
  // find_scale_zp takes any DataType (helpers.rs:101): non-quantized types use (0, 255)
  if (qdtype < LSC_DTYPE_F32 || qdtype > LSC_DTYPE_QINT32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "find_scale_zp: dtype %d", qdtype);
  if (!workspace || workspace_bytes < kFindScaleZpWorkspace ||
      (reinterpret_cast<uintptr_t>(workspace) & 3))
    return set_error(LSC_ERROR_INVALID_ARGUMENT,
                     "find_scale_zp: needs a 4-byte aligned workspace of %u bytes",
                     static_cast<unsigned>(kFindScaleZpWorkspace));
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  uint32_t* ws = static_cast<uint32_t*>(workspace);
  init_minmax_ws<<<1, 1, 0, st>>>(ws);
  if (n == 0) {
    // QuantizationParameters::default(): scale 1, zero point 0 (quantization/scheme.rs:123-127)
    const float one = 1.0f;
    const int32_t zero = 0;
    LSC_CUDA_TRY(cudaMemcpyAsync(scale_out, &one, sizeof(one), cudaMemcpyHostToDevice, st));
    LSC_CUDA_TRY(cudaMemcpyAsync(zp_out, &zero, sizeof(zero), cudaMemcpyHostToDevice, st));
    return LSC_SUCCESS;
  }
  const int grid = grid_for(n, ds->sm_count, 512);
  find_scale_zp_kernel<<<grid, 512, 0, st>>>(x, n, qdtype, symmetric, ws, scale_out, zp_out);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

namespace {
__global__ void fill_default_params(float* scales, int32_t* zps, int64_t rows) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < rows;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    scales[i] = 1.0f;
    zps[i] = 0;
  }
}
}  // namespace

uint64_t find_scale_zp_rows_workspace(int64_t rows) {
  return rows > 0 ? static_cast<uint64_t>(rows) * 12u : 0u;
}

lsc_status launch_find_scale_zp_rows(const float* x, int64_t rows, int64_t cols, int qdtype,
                                     int symmetric, uint32_t* ws, uint64_t ws_bytes,
                                     float* scales, int32_t* zps, cudaStream_t st) {
  if (rows < 0 || cols < 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "find_scale_zp_per_channel: negative size");
  if (rows == 0) return LSC_SUCCESS;
  if (!scales || !zps) return set_error(LSC_ERROR_INVALID_ARGUMENT, "find_scale_zp_per_channel: null output");
  if (cols > 0 && !x) return set_error(LSC_ERROR_INVALID_ARGUMENT, "find_scale_zp_per_channel: null input");
  // find_scale_zp takes any DataType (helpers.rs:101): non-quantized types use (0, 255)
  if (qdtype < LSC_DTYPE_F32 || qdtype > LSC_DTYPE_QINT32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "find_scale_zp_per_channel: dtype %d", qdtype);
  if (!ws || ws_bytes < find_scale_zp_rows_workspace(rows) || (reinterpret_cast<uintptr_t>(ws) & 3))
    return set_error(LSC_ERROR_INVALID_ARGUMENT,
                     "find_scale_zp_per_channel: needs a 4-byte aligned workspace of %llu bytes",
                     static_cast<unsigned long long>(find_scale_zp_rows_workspace(rows)));
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const int fill_grid = grid_for(rows, ds->sm_count, 256);
  if (cols == 0) {
    // QuantizationParameters::default() per channel (quantization/scheme.rs:123-127)
    fill_default_params<<<fill_grid, 256, 0, st>>>(scales, zps, rows);
    LSC_CUDA_TRY(cudaGetLastError());
    return LSC_SUCCESS;
  }
  // Rows longer than 64 Ki elements are split so long channels still fill the GPU.
  const int64_t chunk = cols < 65536 ? cols : 65536;
  const int64_t chunks = (cols + chunk - 1) / chunk;
  if (rows * chunks > INT32_MAX)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "find_scale_zp_per_channel: too many blocks");
  init_minmax_rows<<<fill_grid, 256, 0, st>>>(ws, rows);
  find_scale_zp_rows_kernel<<<static_cast<unsigned>(rows * chunks), 256, 0, st>>>(
      x, rows, cols, chunk, static_cast<int32_t>(chunks), qdtype, symmetric, ws, scales, zps);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

}  // namespace lsc

using namespace lsc;

extern "C" {

lsc_status lsc_quantize_f32(const float* x, void* out, int64_t n, int32_t qdtype, float scale,
                            int32_t zero_point, int32_t rounding, lsc_stream stream) {
  return launch_quantize(x, out, n, qdtype, nullptr, nullptr, scale, zero_point, 1, 1, rounding,
                         static_cast<cudaStream_t>(stream));
}

lsc_status lsc_quantize_f32_per_channel(const float* x, void* out, int64_t n, int32_t qdtype,
                                        const float* scales, const int32_t* zero_points,
                                        int32_t channels, int64_t inner, int32_t rounding,
                                        lsc_stream stream) {
  if (!scales) return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantize_per_channel: null scales");
  return launch_quantize(x, out, n, qdtype, scales, zero_points, 1.0f, 0, channels, inner,
                         rounding, static_cast<cudaStream_t>(stream));
}

lsc_status lsc_dequantize(const void* q, int32_t qdtype, float* out, int64_t n, float scale,
                          int32_t zero_point, lsc_stream stream) {
  return launch_dequantize(q, qdtype, out, n, nullptr, nullptr, scale, zero_point, 1, 1,
                           static_cast<cudaStream_t>(stream));
}

lsc_status lsc_dequantize_per_channel(const void* q, int32_t qdtype, float* out, int64_t n,
                                      const float* scales, const int32_t* zero_points,
                                      int32_t channels, int64_t inner, lsc_stream stream) {
  if (!scales) return set_error(LSC_ERROR_INVALID_ARGUMENT, "dequantize_per_channel: null scales");
  return launch_dequantize(q, qdtype, out, n, scales, zero_points, 1.0f, 0, channels, inner,
                           static_cast<cudaStream_t>(stream));
}

uint64_t lsc_find_scale_zp_workspace_size(void) { return kFindScaleZpWorkspace; }

lsc_status lsc_find_scale_zp_f32(const float* x, int64_t n, int32_t qdtype, int32_t symmetric,
                                 void* workspace, uint64_t workspace_bytes, float* scale_out,
                                 int32_t* zero_point_out, lsc_stream stream) {
  return launch_find_scale_zp(x, n, qdtype, symmetric, workspace, workspace_bytes, scale_out,
                              zero_point_out, static_cast<cudaStream_t>(stream));
}

uint64_t lsc_find_scale_zp_per_channel_workspace_size(int64_t channels) {
  return find_scale_zp_rows_workspace(channels);
}

}  // extern "C"

// ---------------------------------------------------------------------------------------
// Per-channel find_scale_zp for callers that cannot allocate device memory.
//
// Some callers run inside a host runtime that owns all device memory -- a framework whose
// caching allocator has reserved the GPU, or a serving process with a fixed memory budget
// -- and must not call cudaMalloc: it synchronises the device and fails once the owner
// holds the memory.  This variant needs no caller workspace.  Its scratch is a file-scope
// device array of kNoAllocMaxChannels * 12 bytes (192 KiB), which every GPU that loads
// this library holds until the process exits.  The array is reserved when the CUDA module
// of this library is loaded into a context; with lazy module loading (the CUDA 12 default)
// that happens at the first call, so a caller that cannot allocate makes one call per device
// early, before the memory owner has reserved the GPU.
namespace {
constexpr int64_t kNoAllocMaxChannels = 16384;
static __device__ __align__(256) uint32_t g_fsz_noalloc_scratch[3 * kNoAllocMaxChannels];

std::mutex g_noalloc_mu;
struct NoAllocSlot {
  CUcontext ctx = nullptr;  // the context the address below belongs to
  uint32_t* ptr = nullptr;
};
NoAllocSlot g_noalloc_slot[64];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
CtxGetCurrentFn ctx_get_current_fn() {
  static std::once_flag once;
  static CtxGetCurrentFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  });
  return fn;
}

// Device address of the scratch array in the current device's context.  The host-side name
// of a __device__ array is not a device address, so the address is queried with the device
// current and cached together with the context it was taken in: after a cudaDeviceReset the
// primary context (and the module holding the array) is created anew, the cached context no
// longer matches, and the address is looked up again.
lsc_status noalloc_scratch(uint32_t** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return set_error(LSC_ERROR_INVALID_ARGUMENT, "device %d out of range", dev);
  CtxGetCurrentFn get_ctx = ctx_get_current_fn();
  if (!get_ctx) return set_error(LSC_ERROR_DEVICE_ERROR, "cuCtxGetCurrent unavailable");
  CUcontext ctx = nullptr;
  if (get_ctx(&ctx) != CUDA_SUCCESS)
    return set_error(LSC_ERROR_DEVICE_ERROR, "find_scale_zp_per_channel_noalloc: cuCtxGetCurrent failed");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocSlot& slot = g_noalloc_slot[dev];
  if (!ctx || !slot.ptr || slot.ctx != ctx) {
    // the lookup also makes the runtime bind the device's primary context to this thread
    // when none was current yet
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_fsz_noalloc_scratch);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(find_scale_zp scratch)");
    if (!ctx && (get_ctx(&ctx) != CUDA_SUCCESS || !ctx))
      return set_error(LSC_ERROR_DEVICE_ERROR, "find_scale_zp_per_channel_noalloc: no current CUDA context");
    slot.ctx = ctx;
    slot.ptr = static_cast<uint32_t*>(p);
  }
  *out = slot.ptr;
  return LSC_SUCCESS;
}
}  // namespace

extern "C" {

// Same results as lsc_find_scale_zp_per_channel_f32, with the library's own static scratch
// in place of the caller's workspace.  The first call on a device looks up the scratch
// address and, under lazy module loading, loads the module that holds the array (make it
// before any stream capture, and before the memory owner has reserved the device).  Every
// call shares the one array: calls that overlap on the GPU (e.g. on two streams) race; each
// call re-initialises the part it uses, so back-to-back calls are independent.
lsc_status lsc_find_scale_zp_per_channel_f32_noalloc(const float* x, int64_t channels,
                                                     int64_t per_channel, int32_t qdtype,
                                                     int32_t symmetric, float* scales_out,
                                                     int32_t* zero_points_out, lsc_stream stream) {
  if (channels > kNoAllocMaxChannels)
    return set_error(LSC_ERROR_INVALID_ARGUMENT,
                     "find_scale_zp_per_channel_noalloc: %lld channels exceed the static scratch "
                     "limit of %lld; use lsc_find_scale_zp_per_channel_f32 with a workspace",
                     static_cast<long long>(channels), static_cast<long long>(kNoAllocMaxChannels));
  if (channels <= 0) return launch_find_scale_zp_rows(x, channels, per_channel, qdtype, symmetric,
                                                      nullptr, 0, scales_out, zero_points_out,
                                                      static_cast<cudaStream_t>(stream));
  uint32_t* ws = nullptr;
  lsc_status st = noalloc_scratch(&ws);
  if (st) return st;
  return launch_find_scale_zp_rows(x, channels, per_channel, qdtype, symmetric, ws,
                                   sizeof(g_fsz_noalloc_scratch), scales_out, zero_points_out,
                                   static_cast<cudaStream_t>(stream));
}

lsc_status lsc_find_scale_zp_per_channel_f32(const float* x, int64_t channels, int64_t per_channel,
                                             int32_t qdtype, int32_t symmetric, void* workspace,
                                             uint64_t workspace_bytes, float* scales_out,
                                             int32_t* zero_points_out, lsc_stream stream) {
  return launch_find_scale_zp_rows(x, channels, per_channel, qdtype, symmetric,
                                   static_cast<uint32_t*>(workspace), workspace_bytes, scales_out,
                                   zero_points_out, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
