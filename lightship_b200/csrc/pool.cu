// pool.cu -- INT8 NHWC glue of a quantized CNN on the device:
//   quantize_nchw_to_nhwc   f32 NCHW -> int8 NHWC with zero-padded channels, using
//                           quantize_value's arithmetic (quantization/helpers.rs:139-155)
//   maxpool                 MaxPool2d on int8 codes (Pool2d, operator/pooling.rs:383-455);
//                           max commutes with the positive per-tensor dequant scale, so the
//                           codes are pooled directly; padding taps are skipped
//   global average pool     GlobalAvgPool2d (operator/pooling.rs:457-530):
//                           y = ((f32)sum(q) * s_in) / (H*W), then requantized or kept f32
// All HBM-bound: 16 channels (16 bytes) per thread, grids a multiple of the SM count.
#include "epilogue.cuh"
#include "lsc_internal.h"

namespace lsc {
namespace {

__device__ __forceinline__ int32_t sat_i32(float v) {
  if (v != v) return 0;
  if (v >= 2147483648.0f) return INT32_MAX;
  if (v <= -2147483648.0f) return INT32_MIN;
  return __float2int_rz(v);
}

template <int RND>
__device__ __forceinline__ int8_t quantize_i8(float v, float s) {
  const float t = __fdiv_rn(v, s);
  const float r = RND == LSC_ROUND_HALF_EVEN ? rintf(t) : roundf(t);
  int32_t q = sat_i32(r);
  q = q < -128 ? -128 : (q > 127 ? 127 : q);
  return static_cast<int8_t>(q);
}

// one thread per (image, pixel, 16-channel group); reads 16 NCHW planes (strided), writes 16 B
template <int RND>
__global__ void quantize_nchw_to_nhwc_kernel(const float* __restrict__ x, int8_t* __restrict__ y,
                                             int64_t n, int64_t c, int64_t hw, int64_t cp,
                                             float scale) {
  const int64_t groups = cp / 16;
  const int64_t total = n * hw * groups;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t g = i % groups;
    const int64_t pix = (i / groups) % hw;
    const int64_t img = i / (groups * hw);
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t ch = g * 16 + j;
      int8_t q = 0;
      if (ch < c) q = quantize_i8<RND>(__ldg(x + (img * c + ch) * hw + pix), scale);
      w[j >> 2] |= (static_cast<uint32_t>(static_cast<uint8_t>(q))) << (8 * (j & 3));
    }
    reinterpret_cast<uint4*>(y + (img * hw + pix) * cp)[g] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Space-to-depth variant: zero-pad the NCHW input by (ph, pw), then fold each b x b block of
// pixels into channels: out[img, y, x, (dy*b + dx)*C + c] = q(x[img, c, b*y+dy-ph, b*x+dx-pw]).
// A stride-b convolution over the padded input equals a stride-1 convolution over this
// tensor with the filter re-indexed the same way, so a 7x7 stride-2 stem on 3 channels becomes
// a 4x4 stride-1 conv on 12 (stored 16) channels with contiguous, full-sector loads.
template <int RND>
__global__ void quantize_nchw_to_s2d_kernel(const float* __restrict__ x, int8_t* __restrict__ y,
                                            int64_t n, int64_t c, int64_t h, int64_t w,
                                            int64_t ph, int64_t pw, int64_t blk, int64_t hs,
                                            int64_t ws, int64_t cp, float scale) {
  const int64_t groups = cp / 16;
  const int64_t total = n * hs * ws * groups;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t g = i % groups;
    int64_t t = i / groups;
    const int64_t xs = t % ws;
    t /= ws;
    const int64_t ys = t % hs;
    const int64_t img = t / hs;
    uint32_t wd[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t ch = g * 16 + j;
      int8_t q = 0;
      if (ch < blk * blk * c) {
        const int64_t cc = ch % c, blkidx = ch / c;
        const int64_t iy = ys * blk + blkidx / blk - ph, ix = xs * blk + blkidx % blk - pw;
        if (iy >= 0 && iy < h && ix >= 0 && ix < w)
          q = quantize_i8<RND>(__ldg(x + ((img * c + cc) * h + iy) * w + ix), scale);
      }
      wd[j >> 2] |= (static_cast<uint32_t>(static_cast<uint8_t>(q))) << (8 * (j & 3));
    }
    reinterpret_cast<uint4*>(y + ((img * hs + ys) * ws + xs) * cp)[g] = make_uint4(wd[0], wd[1], wd[2], wd[3]);
  }
}

__device__ __forceinline__ uint32_t vmax_s8x4(uint32_t a, uint32_t b) { return __vmaxs4(a, b); }

__global__ void maxpool_i8_kernel(const int8_t* __restrict__ x, int8_t* __restrict__ y, int64_t n,
                                  int64_t h, int64_t w, int64_t c, int64_t oh, int64_t ow, int kh,
                                  int kw, int sh, int sw, int ph, int pw) {
  const int64_t groups = c / 16;
  const int64_t total = n * oh * ow * groups;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t g = i % groups;
    int64_t t = i / groups;
    const int64_t ox = t % ow;
    t /= ow;
    const int64_t oy = t % oh;
    const int64_t img = t / oh;
    uint4 m = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);  // -128 x 16
    for (int r = 0; r < kh; ++r) {
      const int64_t iy = oy * sh - ph + r;
      if (iy < 0 || iy >= h) continue;
      for (int s = 0; s < kw; ++s) {
        const int64_t ix = ox * sw - pw + s;
        if (ix < 0 || ix >= w) continue;
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(x + ((img * h + iy) * w + ix) * c) + g);
        m.x = vmax_s8x4(m.x, v.x);
        m.y = vmax_s8x4(m.y, v.y);
        m.z = vmax_s8x4(m.z, v.z);
        m.w = vmax_s8x4(m.w, v.w);
      }
    }
    reinterpret_cast<uint4*>(y + ((img * oh + oy) * ow + ox) * c)[g] = m;
  }
}

// one warp per (image, 32-channel slab): lanes own channels, loop over pixels
template <int RND>
__global__ void avgpool_i8_kernel(const int8_t* __restrict__ x, int64_t n, int64_t hw, int64_t c,
                                  float s_in, float s_out, int8_t* __restrict__ y_i8,
                                  float* __restrict__ y_f32) {
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  const int64_t slabs = (c + 31) / 32;
  for (int64_t wi = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) + threadIdx.x / 32;
       wi < n * slabs; wi += warps) {
    const int64_t img = wi / slabs;
    const int64_t ch = (wi % slabs) * 32 + (threadIdx.x & 31);
    if (ch >= c) continue;
    int32_t sum = 0;
    const int8_t* p = x + img * hw * c + ch;
    for (int64_t q = 0; q < hw; ++q) sum += p[q * c];
    const float v = __fdiv_rn(__fmul_rn(__int2float_rn(sum), s_in), static_cast<float>(hw));
    if (y_f32) y_f32[img * c + ch] = v;
    if (y_i8) y_i8[img * c + ch] = quantize_i8<RND>(v, s_out);
  }
}

int grid_p(int64_t n, int sm_count) {
  int64_t g = (n + 255) / 256;
  const int64_t cap = static_cast<int64_t>(sm_count) * 8;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

lsc_status launch_quantize_nchw_to_nhwc_i8(const float* x, int8_t* y, int64_t n, int64_t c,
                                           int64_t hw, int64_t cp, float scale, int rounding,
                                           cudaStream_t st) {
  if (cp % 16 != 0 || cp < c)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantize NCHW->NHWC: stored channels must be a multiple of 16 and >= C");
  if (reinterpret_cast<uintptr_t>(y) & 15) return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantize NCHW->NHWC: output must be 16-byte aligned");
  const int64_t total = n * hw * (cp / 16);
  if (total == 0) return LSC_SUCCESS;
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (rounding == LSC_ROUND_HALF_EVEN)
    quantize_nchw_to_nhwc_kernel<LSC_ROUND_HALF_EVEN><<<grid_p(total, ds->sm_count), 256, 0, st>>>(x, y, n, c, hw, cp, scale);
  else
    quantize_nchw_to_nhwc_kernel<LSC_ROUND_HALF_AWAY><<<grid_p(total, ds->sm_count), 256, 0, st>>>(x, y, n, c, hw, cp, scale);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

lsc_status launch_quantize_nchw_to_s2d_i8(const float* x, int8_t* y, int64_t n, int64_t c, int64_t h,
                                          int64_t w, int64_t ph, int64_t pw, int64_t ph_end, int64_t pw_end,
                                          int64_t blk, int64_t cp, float scale, int rounding, cudaStream_t st) {
  if (blk < 2 || ph < 0 || pw < 0 || ph_end < 0 || pw_end < 0)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "space-to-depth: bad block/padding");
  if (cp % 16 != 0 || cp < blk * blk * c)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "space-to-depth: stored channels must be a multiple of 16 and >= %lld",
                     (long long)(blk * blk * c));
  if ((h + ph + ph_end) % blk || (w + pw + pw_end) % blk)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "space-to-depth: padded size not divisible by the block");
  if (reinterpret_cast<uintptr_t>(y) & 15) return set_error(LSC_ERROR_INVALID_ARGUMENT, "space-to-depth: output must be 16-byte aligned");
  const int64_t hs = (h + ph + ph_end) / blk, ws = (w + pw + pw_end) / blk;
  const int64_t total = n * hs * ws * (cp / 16);
  if (total == 0) return LSC_SUCCESS;
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  if (rounding == LSC_ROUND_HALF_EVEN)
    quantize_nchw_to_s2d_kernel<LSC_ROUND_HALF_EVEN><<<grid_p(total, ds->sm_count), 256, 0, st>>>(
        x, y, n, c, h, w, ph, pw, blk, hs, ws, cp, scale);
  else
    quantize_nchw_to_s2d_kernel<LSC_ROUND_HALF_AWAY><<<grid_p(total, ds->sm_count), 256, 0, st>>>(
        x, y, n, c, h, w, ph, pw, blk, hs, ws, cp, scale);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

lsc_status launch_maxpool_i8(const int8_t* x, int8_t* y, int64_t n, int64_t h, int64_t w, int64_t c,
                             int64_t oh, int64_t ow, int kh, int kw, int sh, int sw, int ph, int pw,
                             cudaStream_t st) {
  if (c % 16 != 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "maxpool: channels must be a multiple of 16");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "maxpool: tensors must be 16-byte aligned");
  const int64_t total = n * oh * ow * (c / 16);
  if (total == 0) return LSC_SUCCESS;
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  maxpool_i8_kernel<<<grid_p(total, ds->sm_count), 256, 0, st>>>(x, y, n, h, w, c, oh, ow, kh, kw, sh, sw, ph, pw);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

lsc_status launch_avgpool_i8(const int8_t* x, int64_t n, int64_t hw, int64_t c, float s_in, float s_out,
                             int rounding, int8_t* y_i8, float* y_f32, cudaStream_t st) {
  if (n * c == 0) return LSC_SUCCESS;
  if (hw <= 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "global avgpool: empty spatial extent");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const int64_t warps = n * ((c + 31) / 32);
  const int grid = grid_p(warps * 32, ds->sm_count);
  if (rounding == LSC_ROUND_HALF_EVEN)
    avgpool_i8_kernel<LSC_ROUND_HALF_EVEN><<<grid, 256, 0, st>>>(x, n, hw, c, s_in, s_out, y_i8, y_f32);
  else
    avgpool_i8_kernel<LSC_ROUND_HALF_AWAY><<<grid, 256, 0, st>>>(x, n, hw, c, s_in, s_out, y_i8, y_f32);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

}  // namespace lsc
