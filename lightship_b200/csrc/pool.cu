// pool.cu -- INT8 NHWC glue of a quantized CNN on the device:
//   quantize_nchw_to_nhwc   f32 NCHW -> int8 NHWC with zero-padded channels, using
//                           quantize_value's arithmetic (quantization/helpers.rs:139-155)
//   maxpool                 MaxPool2d on int8 codes (Pool2d, operator/pooling.rs:383-455);
//                           max commutes with the positive per-tensor dequant scale, so the
//                           codes are pooled directly; padding taps are skipped
//   global average pool     GlobalAvgPool2d (operator/pooling.rs:457-530):
//                           y = ((f32)sum(q) * s_in) / (H*W), then requantized or kept f32
// All HBM-bound: 16 channels (16 bytes) per thread, grids a multiple of the SM count.
#include <math.h>

#include <cmath>

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

// grid (pixel blocks, image): one thread per (pixel, 16-channel group), pixel-major so a
// warp's reads of one NCHW plane are consecutive floats; writes 16 B.  32-bit index math
// within an image (the launcher checks the image size).
template <int RND>
__global__ void quantize_nchw_to_nhwc_kernel(const float* __restrict__ x, int8_t* __restrict__ y,
                                             int c, int hw, int cp, float scale, float inv_s) {
  griddep_wait();  // launched as a dependent kernel: inputs and outputs are settled from here on
  griddep_launch_dependents();
  const int groups = cp >> 4;
  const int img = blockIdx.y;
  const float* xi = x + static_cast<size_t>(img) * c * hw;
  int8_t* yi = y + static_cast<size_t>(img) * hw * cp;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hw * groups; i += gridDim.x * blockDim.x) {
    const int pix = i % hw;
    const int g = i / hw;
    uint32_t w[4] = {0, 0, 0, 0};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int ch = g * 16 + j;
      int8_t q = 0;
      if (ch < c) q = static_cast<int8_t>(requant_one<RND>(__ldg(xi + static_cast<size_t>(ch) * hw + pix), scale, inv_s));
      w[j >> 2] |= (static_cast<uint32_t>(static_cast<uint8_t>(q))) << (8 * (j & 3));
    }
    reinterpret_cast<uint4*>(yi + static_cast<size_t>(pix) * cp)[g] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Space-to-depth variant: zero-pad the NCHW input by (ph, pw), then fold each b x b block of
// pixels into channels: out[img, y, x, (dy*b + dx)*C + c] = q(x[img, c, b*y+dy-ph, b*x+dx-pw]).
// A stride-b convolution over the padded input equals a stride-1 convolution over this
// tensor with the filter re-indexed the same way, so a 7x7 stride-2 stem on 3 channels becomes
// a 4x4 stride-1 conv on 12 (stored 16) channels with contiguous, full-sector loads.
// grid (column blocks, output row, image): one thread per (output column, 16-channel group).
template <int RND>
__global__ void quantize_nchw_to_s2d_kernel(const float* __restrict__ x, int8_t* __restrict__ y,
                                            int c, int h, int w, int ph, int pw, int blk, int hs,
                                            int ws, int cp, float scale, float inv_s) {
  griddep_wait();  // launched as a dependent kernel: inputs and outputs are settled from here on
  griddep_launch_dependents();
  const int groups = cp >> 4;
  const int ys = blockIdx.y, img = blockIdx.z;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= ws * groups) return;
  const int g = i % groups;
  const int xs = i / groups;
  const float* xi = x + static_cast<size_t>(img) * c * h * w;
  // channel g*16 + j is input channel cc of block position (dy, dx) (channel = (dy*blk + dx)*C + cc)
  const int bi0 = (g * 16) / c;
  int cc = g * 16 - bi0 * c, dy = bi0 / blk, dx = bi0 - dy * blk;
  uint32_t wd[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    int8_t q = 0;
    if (dy < blk) {
      const int iy = ys * blk + dy - ph, ix = xs * blk + dx - pw;
      if (iy >= 0 && iy < h && ix >= 0 && ix < w)
        q = static_cast<int8_t>(requant_one<RND>(__ldg(xi + (static_cast<size_t>(cc) * h + iy) * w + ix), scale, inv_s));
    }
    wd[j >> 2] |= (static_cast<uint32_t>(static_cast<uint8_t>(q))) << (8 * (j & 3));
    if (++cc == c) {
      cc = 0;
      if (++dx == blk) {
        dx = 0;
        ++dy;
      }
    }
  }
  reinterpret_cast<uint4*>(y + ((static_cast<size_t>(img) * hs + ys) * ws + xs) * cp)[g] =
      make_uint4(wd[0], wd[1], wd[2], wd[3]);
}

// The same for the CNN stem's case, C = 3 input channels, 2x2 blocks, 16 stored channels,
// image width a multiple of 4.  grid (1, output row, image), 128 threads, 24 * w bytes of
// dynamic shared memory: the block first stages its two input rows of the three channels
// with 16-byte loads (rows outside the image as zeros), then each thread builds whole 16-byte
// output pixels from shared memory (channel j = (dy * 2 + dx) * 3 + c, bytes 12-15 zero; a
// padding tap quantizes 0, which is code 0).  Reading the rows whole, instead of each thread
// gathering its twelve pixels with scalar loads, keeps the kernel at HBM speed.
template <int RND>
__global__ void __launch_bounds__(128) quantize_nchw_to_s2d_c3b2_kernel(const float* __restrict__ x,
                                                                        int8_t* __restrict__ y, int h, int w,
                                                                        int ph, int pw, int hs, int ws,
                                                                        float scale, float inv_s) {
  extern __shared__ float srow[];  // [dy * 3 + c][w]
  griddep_wait();  // launched as a dependent kernel: inputs and outputs are settled from here on
  griddep_launch_dependents();
  const int ys = blockIdx.y, img = blockIdx.z;
  const int plane = h * w;
  const float* xi = x + static_cast<size_t>(img) * 3 * plane;
  const int w4 = w >> 2;
  for (int i = threadIdx.x; i < 6 * w4; i += blockDim.x) {
    const int r = i / w4, q = i - r * w4;
    const int dy = r / 3, cc = r - dy * 3;
    const int iy = ys * 2 + dy - ph;
    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (iy >= 0 && iy < h) v = __ldg(reinterpret_cast<const float4*>(xi + cc * plane + iy * w) + q);
    reinterpret_cast<float4*>(srow + r * w)[q] = v;
  }
  __syncthreads();
  for (int xs = threadIdx.x; xs < ws; xs += blockDim.x) {
    uint32_t wd[4] = {0, 0, 0, 0};
#pragma unroll
    for (int dy = 0; dy < 2; ++dy) {
#pragma unroll
      for (int dx = 0; dx < 2; ++dx) {
        const int ix = xs * 2 + dx - pw;
        if (ix < 0 || ix >= w) continue;
#pragma unroll
        for (int cc = 0; cc < 3; ++cc) {
          const int j = (dy * 2 + dx) * 3 + cc;
          const int32_t q = requant_one<RND>(srow[(dy * 3 + cc) * w + ix], scale, inv_s);
          wd[j >> 2] |= (static_cast<uint32_t>(q) & 0xFFu) << (8 * (j & 3));
        }
      }
    }
    reinterpret_cast<uint4*>(y + ((static_cast<size_t>(img) * hs + ys) * ws + xs) * 16)[0] =
        make_uint4(wd[0], wd[1], wd[2], wd[3]);
  }
}

__device__ __forceinline__ uint32_t vmax_s8x4(uint32_t a, uint32_t b) { return __vmaxs4(a, b); }

// grid (column blocks, output row, image): one thread per (output column, 16-channel group),
// group-major so a warp's 16-byte loads of one tap are contiguous.  KH/KW > 0 fix the window
// at compile time (3x3 and 2x2); 0 takes it from kh/kw.
template <int KH, int KW>
__global__ void maxpool_i8_kernel(const int8_t* __restrict__ x, int8_t* __restrict__ y, int h, int w,
                                  int c, int oh, int ow, int kh, int kw, int sh, int sw, int ph, int pw) {
  griddep_wait();  // launched as a dependent kernel: inputs and outputs are settled from here on
  griddep_launch_dependents();
  const int groups = c >> 4;
  const int oy = blockIdx.y, img = blockIdx.z;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= ow * groups) return;
  const int g = i % groups;
  const int ox = i / groups;
  const int nh = KH > 0 ? KH : kh, nw = KW > 0 ? KW : kw;
  const uint4* xi = reinterpret_cast<const uint4*>(x + static_cast<size_t>(img) * h * w * c) + g;
  uint4 m = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);  // -128 x 16
#pragma unroll
  for (int r = 0; r < nh; ++r) {
    const int iy = oy * sh - ph + r;
    if (iy < 0 || iy >= h) continue;
#pragma unroll
    for (int s = 0; s < nw; ++s) {
      const int ix = ox * sw - pw + s;
      if (ix < 0 || ix >= w) continue;
      const uint4 v = __ldg(xi + (iy * w + ix) * groups);
      m.x = vmax_s8x4(m.x, v.x);
      m.y = vmax_s8x4(m.y, v.y);
      m.z = vmax_s8x4(m.z, v.z);
      m.w = vmax_s8x4(m.w, v.w);
    }
  }
  reinterpret_cast<uint4*>(y + ((static_cast<size_t>(img) * oh + oy) * ow + ox) * c)[g] = m;
}

// one warp per (image, 32-channel slab): lanes own channels, loop over pixels
template <int RND>
__global__ void avgpool_i8_kernel(const int8_t* __restrict__ x, int64_t n, int64_t hw, int64_t c,
                                  float s_in, float s_out, int8_t* __restrict__ y_i8,
                                  float* __restrict__ y_f32) {
  griddep_wait();  // launched as a dependent kernel: inputs and outputs are settled from here on
  griddep_launch_dependents();
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

// MaxPool2d on f32 NCHW (Pool2d::max_pool2d, operator/pooling.rs): the max over the window's
// in-bounds taps (padding taps take no part), one thread per output element.
__global__ void maxpool_f32_nchw_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t planes,
                                        int h, int w, int oh, int ow, int kh, int kw, int sh, int sw, int ph,
                                        int pw) {
  griddep_wait();  // launched as a dependent kernel: inputs and outputs are settled from here on
  griddep_launch_dependents();
  const int64_t total = planes * oh * ow;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int ox = static_cast<int>(i % ow);
    const int oy = static_cast<int>((i / ow) % oh);
    const int64_t plane = i / (static_cast<int64_t>(ow) * oh);
    const float* xp = x + plane * h * w;
    float m = -INFINITY;
    for (int r = 0; r < kh; ++r) {
      const int iy = oy * sh - ph + r;
      if (iy < 0 || iy >= h) continue;
      for (int c = 0; c < kw; ++c) {
        const int ix = ox * sw - pw + c;
        if (ix < 0 || ix >= w) continue;
        m = fmaxf(m, __ldg(xp + static_cast<int64_t>(iy) * w + ix));
      }
    }
    y[i] = m;
  }
}

// GlobalAvgPool2d on f32 NCHW (operator/pooling.rs:457-490): (sum of the plane) / (H*W), one
// warp per (n, c) plane; the sum is tree-ordered (the reference sums in sequence).
__global__ void avgpool_f32_nchw_kernel(const float* __restrict__ x, float* __restrict__ y, int64_t planes,
                                        int64_t hw) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t p = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); p < planes;
       p += warps) {
    const float* xp = x + p * hw;
    float acc = 0.0f;
    for (int64_t i = lane; i < hw; i += 32) acc = __fadd_rn(acc, __ldg(xp + i));
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if (lane == 0) y[p] = __fdiv_rn(acc, static_cast<float>(hw));
  }
}

}  // namespace

lsc_status launch_maxpool_f32(const float* x, float* y, int64_t n, int64_t c, int64_t h, int64_t w, int64_t oh,
                              int64_t ow, int kh, int kw, int sh, int sw, int ph, int pw, cudaStream_t st) {
  const int64_t total = n * c * oh * ow;
  if (total == 0) return LSC_SUCCESS;
  if (h > INT32_MAX || w > INT32_MAX) return set_error(LSC_ERROR_INVALID_ARGUMENT, "maxpool: image too large");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  int64_t g = (total + 255) / 256;
  if (g > static_cast<int64_t>(ds->sm_count) * 8) g = static_cast<int64_t>(ds->sm_count) * 8;
  LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, maxpool_f32_nchw_kernel, dim3(static_cast<unsigned>(g)),
                                dim3(256), 0, st, x, y, n * c, static_cast<int>(h), static_cast<int>(w),
                                static_cast<int>(oh), static_cast<int>(ow), kh, kw, sh, sw, ph, pw));
  return LSC_SUCCESS;
}

lsc_status launch_avgpool_f32(const float* x, float* y, int64_t n, int64_t c, int64_t hw, cudaStream_t st) {
  const int64_t planes = n * c;
  if (planes == 0) return LSC_SUCCESS;
  if (hw <= 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "global avgpool: empty spatial extent");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  int64_t g = (planes + 7) / 8;
  if (g > static_cast<int64_t>(ds->sm_count) * 8) g = static_cast<int64_t>(ds->sm_count) * 8;
  LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, avgpool_f32_nchw_kernel, dim3(static_cast<unsigned>(g)),
                                dim3(256), 0, st, x, y, planes, hw));
  return LSC_SUCCESS;
}

// RN(1 / s) when s and its reciprocal are normal floats (the reciprocal requantization's
// precondition), else 0, which makes every element take the division.
float reciprocal_or_zero(float s) {
  const float inv = 1.0f / s;
  return (std::isnormal(s) && std::isnormal(inv)) ? inv : 0.0f;
}

lsc_status launch_quantize_nchw_to_nhwc_i8(const float* x, int8_t* y, int64_t n, int64_t c,
                                           int64_t hw, int64_t cp, float scale, int rounding,
                                           cudaStream_t st) {
  if (cp % 16 != 0 || cp < c)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantize NCHW->NHWC: stored channels must be a multiple of 16 and >= C");
  if (reinterpret_cast<uintptr_t>(y) & 15) return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantize NCHW->NHWC: output must be 16-byte aligned");
  const int64_t per_img = hw * (cp / 16);
  if (n == 0 || per_img == 0) return LSC_SUCCESS;
  if (n > 65535 || hw * cp > INT32_MAX || c * hw > INT32_MAX)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantize NCHW->NHWC: batch or image too large");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const float inv_s = reciprocal_or_zero(scale);
  int64_t bx = (per_img + 255) / 256;
  const int64_t cap = (static_cast<int64_t>(ds->sm_count) * 8 + n - 1) / n;
  if (bx > cap) bx = cap;
  const dim3 grid(static_cast<unsigned>(bx < 1 ? 1 : bx), static_cast<unsigned>(n));
  if (rounding == LSC_ROUND_HALF_EVEN)
    LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, quantize_nchw_to_nhwc_kernel<LSC_ROUND_HALF_EVEN>, grid, dim3(256), 0, st,
                                  x, y, static_cast<int>(c), static_cast<int>(hw), static_cast<int>(cp), scale, inv_s));
  else
    LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, quantize_nchw_to_nhwc_kernel<LSC_ROUND_HALF_AWAY>, grid, dim3(256), 0, st,
                                  x, y, static_cast<int>(c), static_cast<int>(hw), static_cast<int>(cp), scale, inv_s));
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
  const int64_t per_row = ws * (cp / 16);
  if (n == 0 || hs == 0 || per_row == 0) return LSC_SUCCESS;
  if (n > 65535 || hs > 65535 || c * h * w > INT32_MAX || ws * cp > INT32_MAX || blk > 64)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "space-to-depth: batch or image too large");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const dim3 grid(static_cast<unsigned>((per_row + 127) / 128), static_cast<unsigned>(hs), static_cast<unsigned>(n));
  const int ic = static_cast<int>(c), ih = static_cast<int>(h), iw = static_cast<int>(w);
  const float inv_s = reciprocal_or_zero(scale);
  if (c == 3 && blk == 2 && cp == 16 && w % 4 == 0 && w <= 2048 &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const dim3 g2(1u, static_cast<unsigned>(hs), static_cast<unsigned>(n));
    const size_t smem = static_cast<size_t>(24 * w);
    if (rounding == LSC_ROUND_HALF_EVEN)
      LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, quantize_nchw_to_s2d_c3b2_kernel<LSC_ROUND_HALF_EVEN>, g2,
                                    dim3(128), smem, st, x, y, ih, iw, static_cast<int>(ph), static_cast<int>(pw),
                                    static_cast<int>(hs), static_cast<int>(ws), scale, inv_s));
    else
      LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, quantize_nchw_to_s2d_c3b2_kernel<LSC_ROUND_HALF_AWAY>, g2,
                                    dim3(128), smem, st, x, y, ih, iw, static_cast<int>(ph), static_cast<int>(pw),
                                    static_cast<int>(hs), static_cast<int>(ws), scale, inv_s));
    LSC_CUDA_TRY(cudaGetLastError());
    return LSC_SUCCESS;
  }
  if (rounding == LSC_ROUND_HALF_EVEN)
    LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, quantize_nchw_to_s2d_kernel<LSC_ROUND_HALF_EVEN>, grid, dim3(128),
                                  0, st, x, y, ic, ih, iw, static_cast<int>(ph), static_cast<int>(pw),
                                  static_cast<int>(blk), static_cast<int>(hs), static_cast<int>(ws),
                                  static_cast<int>(cp), scale, inv_s));
  else
    LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, quantize_nchw_to_s2d_kernel<LSC_ROUND_HALF_AWAY>, grid, dim3(128),
                                  0, st, x, y, ic, ih, iw, static_cast<int>(ph), static_cast<int>(pw),
                                  static_cast<int>(blk), static_cast<int>(hs), static_cast<int>(ws),
                                  static_cast<int>(cp), scale, inv_s));
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

lsc_status launch_maxpool_i8(const int8_t* x, int8_t* y, int64_t n, int64_t h, int64_t w, int64_t c,
                             int64_t oh, int64_t ow, int kh, int kw, int sh, int sw, int ph, int pw,
                             cudaStream_t st) {
  if (c % 16 != 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "maxpool: channels must be a multiple of 16");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "maxpool: tensors must be 16-byte aligned");
  const int64_t per_row = ow * (c / 16);
  if (n == 0 || oh == 0 || per_row == 0) return LSC_SUCCESS;
  if (n > 65535 || oh > 65535 || h * w * c > INT32_MAX || oh * ow * c > INT32_MAX)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "maxpool: batch or image too large");
  DeviceState* ds = current_device_state();
  if (!ds) return LSC_ERROR_DEVICE_ERROR;
  const dim3 grid(static_cast<unsigned>((per_row + 127) / 128), static_cast<unsigned>(oh), static_cast<unsigned>(n));
  const int ih = static_cast<int>(h), iw = static_cast<int>(w), ic = static_cast<int>(c);
  const int ioh = static_cast<int>(oh), iow = static_cast<int>(ow);
  if (kh == 3 && kw == 3)
    LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, maxpool_i8_kernel<3, 3>, grid, dim3(128), 0, st, x, y, ih, iw, ic,
                                  ioh, iow, kh, kw, sh, sw, ph, pw));
  else if (kh == 2 && kw == 2)
    LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, maxpool_i8_kernel<2, 2>, grid, dim3(128), 0, st, x, y, ih, iw, ic,
                                  ioh, iow, kh, kw, sh, sw, ph, pw));
  else
    LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, maxpool_i8_kernel<0, 0>, grid, dim3(128), 0, st, x, y, ih, iw, ic,
                                  ioh, iow, kh, kw, sh, sw, ph, pw));
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
    LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, avgpool_i8_kernel<LSC_ROUND_HALF_EVEN>, dim3(grid), dim3(256), 0,
                                  st, x, n, hw, c, s_in, s_out, y_i8, y_f32));
  else
    LSC_CUDA_TRY(launch_dependent(ds->overlap_launches, avgpool_i8_kernel<LSC_ROUND_HALF_AWAY>, dim3(grid), dim3(256), 0,
                                  st, x, n, hw, c, s_in, s_out, y_i8, y_f32));
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

}  // namespace lsc
