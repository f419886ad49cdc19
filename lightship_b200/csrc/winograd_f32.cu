// winograd_f32.cu -- FP32 Conv2d 3x3, stride 1, dilation 1 as Winograd F(2x2, 3x3)
// (the reference's WinogradConv2d, lightship-core/src/cpu/winograd_conv2d.rs:50-397:
// Lavin & Gray, "Fast Algorithms for Convolutional Neural Networks", CVPR 2016).
//
// Every 2x2 output tile t of image n reads a 4x4 input patch d (origin 2*ty - pad_h,
// 2*tx - pad_w, zero outside the image) and is
//     Y = A^T [ sum_c (G g_c G^T) (.) (B^T d_c B) ] A
// with B^T = [1 0 -1 0; 0 1 1 0; 0 -1 1 0; 0 1 0 -1], G = [1 0 0; .5 .5 .5; .5 -.5 .5; 0 0 1],
// A^T = [1 1 1 0; 0 1 -1 -1].  The sum over channels of the elementwise product is, for each
// of the 16 positions xi of the 4x4 transformed tile, a GEMM
//     M_xi[T, Cout] = V_xi[T, C] . U_xi[Cout, C]^T,
// run as one batched split-TF32 tensor-core GEMM (contraction_tf32.cu, 16 batches).
//   * filter transform U = G g G^T: once at compile, on the host (backend_conv.cpp)
//   * input transform (this file): NCHW input -> V_hi / V_lo [16][T][Cp], the split-TF32
//     halves the GEMM loads by TMA (channels padded to Cp = a multiple of 4 with zeros)
//   * output transform (this file): M [16][T][Cout] -> Y = A^T m A, + bias, activation,
//     written NCHW
// 2.25x fewer multiplications than the direct convolution, paid for with the transforms'
// HBM traffic (V is 16/4 = 4x the input per half, M 4x the output).
#include "epilogue.cuh"
#include "lsc_internal.h"

namespace lsc {
namespace {

constexpr int kWT = 16;  // tiles per block along the width
constexpr int kWC = 32;  // channels per block
constexpr int kInCols = 2 * kWT + 2;
constexpr int kInStride = 4 * kInCols + 1;   // odd: conflict-free across channels
constexpr int kOutStride = 2 * 2 * kWT + 1;  // 2 rows x 32 columns per channel, odd

__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = __fsub_rn(x, hi);
}

__device__ __forceinline__ float act_rt_w(float x, int act) {
  switch (act) {
    case LSC_ACT_RELU: return act_relu(x);
    case LSC_ACT_RELU6: return act_relu6(x);
    case LSC_ACT_SILU: return act_silu(x);
    case LSC_ACT_GELU: return act_gelu(x);
    default: return x;
  }
}

// grid (ceil(tw / 16), n * th, ceil(cp / 32)), 256 threads.  The block stages the 4-row,
// 34-column input band of its 16 tiles for 32 channels (coalesced along the width), then each
// thread transforms (tile, channel) pairs with the channel fastest, so the 16 V planes are
// written as 128-byte rows.
__global__ void __launch_bounds__(256) winograd_input_kernel(const float* __restrict__ x, int c, int h, int w,
                                                             int ph, int pw, int th, int tw, int cp,
                                                             int64_t tiles, float* __restrict__ vhi,
                                                             float* __restrict__ vlo) {
  __shared__ float s[kWC * kInStride];
  const int tx0 = blockIdx.x * kWT;
  const int img = blockIdx.y / th, ty = blockIdx.y - img * th;
  const int c0 = blockIdx.z * kWC;
  const int y0 = 2 * ty - ph, x0 = 2 * tx0 - pw;
  for (int i = threadIdx.x; i < kWC * 4 * kInCols; i += blockDim.x) {
    const int col = i % kInCols;
    const int r = (i / kInCols) & 3;
    const int cc = i / (4 * kInCols);
    const int gy = y0 + r, gx = x0 + col, ch = c0 + cc;
    float v = 0.0f;
    if (ch < c && gy >= 0 && gy < h && gx >= 0 && gx < w)
      v = __ldg(x + ((static_cast<int64_t>(img) * c + ch) * h + gy) * w + gx);
    s[cc * kInStride + r * kInCols + col] = v;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kWT * kWC; i += blockDim.x) {
    const int cc = i % kWC, tl = i / kWC;
    const int tx = tx0 + tl, ch = c0 + cc;
    if (tx >= tw || ch >= cp) continue;
    const float* d = s + cc * kInStride + 2 * tl;
    float b[4][4];  // B^T d
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float d0 = d[j], d1 = d[kInCols + j], d2 = d[2 * kInCols + j], d3 = d[3 * kInCols + j];
      b[0][j] = __fsub_rn(d0, d2);
      b[1][j] = __fadd_rn(d1, d2);
      b[2][j] = __fsub_rn(d2, d1);
      b[3][j] = __fsub_rn(d1, d3);
    }
    const int64_t t = static_cast<int64_t>(blockIdx.y) * tw + tx;  // (img * th + ty) * tw + tx
    float v[16];
#pragma unroll
    for (int r = 0; r < 4; ++r) {  // (B^T d) B
      v[4 * r + 0] = __fsub_rn(b[r][0], b[r][2]);
      v[4 * r + 1] = __fadd_rn(b[r][1], b[r][2]);
      v[4 * r + 2] = __fsub_rn(b[r][2], b[r][1]);
      v[4 * r + 3] = __fsub_rn(b[r][1], b[r][3]);
    }
#pragma unroll
    for (int xi = 0; xi < 16; ++xi) {
      float hi, lo;
      split_tf32(v[xi], hi, lo);
      const int64_t o = (xi * tiles + t) * cp + ch;
      vhi[o] = hi;
      if (vlo) vlo[o] = lo;
    }
  }
}

// grid (ceil(tw / 16), n * th, ceil(cout / 32)), 256 threads.  Each thread inverse-transforms
// (tile, output channel) pairs with the channel fastest (the 16 M planes read as 128-byte
// rows), adds the bias and applies the activation, and the block writes its 2 output rows x
// 32 columns per channel back NCHW.
__global__ void __launch_bounds__(256) winograd_output_kernel(const float* __restrict__ m, int64_t tiles, int cout,
                                                              int th, int tw, int oh, int ow,
                                                              const float* __restrict__ bias, int act,
                                                              float* __restrict__ y) {
  __shared__ float s[kWC * kOutStride];
  const int tx0 = blockIdx.x * kWT;
  const int img = blockIdx.y / th, ty = blockIdx.y - img * th;
  const int c0 = blockIdx.z * kWC;
  for (int i = threadIdx.x; i < kWT * kWC; i += blockDim.x) {
    const int cc = i % kWC, tl = i / kWC;
    const int tx = tx0 + tl, co = c0 + cc;
    if (tx >= tw || co >= cout) continue;
    const int64_t t = static_cast<int64_t>(blockIdx.y) * tw + tx;
    float v[16];
#pragma unroll
    for (int xi = 0; xi < 16; ++xi) v[xi] = __ldg(m + (xi * tiles + t) * cout + co);
    float a[2][4];  // A^T m
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      a[0][j] = __fadd_rn(__fadd_rn(v[j], v[4 + j]), v[8 + j]);
      a[1][j] = __fsub_rn(__fsub_rn(v[4 + j], v[8 + j]), v[12 + j]);
    }
    const float bv = bias ? __ldg(bias + co) : 0.0f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {  // (A^T m) A
      float y0 = __fadd_rn(__fadd_rn(a[r][0], a[r][1]), a[r][2]);
      float y1 = __fsub_rn(__fsub_rn(a[r][1], a[r][2]), a[r][3]);
      if (bias) {
        y0 = __fadd_rn(y0, bv);
        y1 = __fadd_rn(y1, bv);
      }
      s[cc * kOutStride + r * (2 * kWT) + 2 * tl] = act_rt_w(y0, act);
      s[cc * kOutStride + r * (2 * kWT) + 2 * tl + 1] = act_rt_w(y1, act);
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < kWC * 2 * 2 * kWT; i += blockDim.x) {
    const int col = i % (2 * kWT);
    const int r = (i / (2 * kWT)) & 1;
    const int cc = i / (4 * kWT);
    const int co = c0 + cc, oy = 2 * ty + r, ox = 2 * tx0 + col;
    if (co < cout && oy < oh && ox < ow)
      y[((static_cast<int64_t>(img) * cout + co) * oh + oy) * ow + ox] = s[cc * kOutStride + r * (2 * kWT) + col];
  }
}

}  // namespace

int64_t winograd_f32_scratch_floats(const ConvGeometry& g, int64_t cp, bool split) {
  const int64_t th = (g.oh + 1) / 2, tw = (g.ow + 1) / 2;
  const int64_t tiles = g.n * th * tw;
  return 16 * tiles * cp * (split ? 2 : 1) + 16 * tiles * g.c_out;
}

lsc_status launch_conv_winograd_f32(const float* x_nchw, const float* u_hi, const float* u_lo,
                                    const ConvGeometry& g, int64_t cp, const float* bias, int act,
                                    float* out_nchw, float* scratch, bool split, cudaStream_t stream) {
  if (g.kh != 3 || g.kw != 3 || g.sh != 1 || g.sw != 1 || g.dh != 1 || g.dw != 1)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "winograd_f32: 3x3, stride 1, dilation 1 only");
  if (g.n < 0 || g.c <= 0 || g.h <= 0 || g.w <= 0 || g.c_out <= 0 || cp < g.c || cp % 4 != 0)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "winograd_f32: bad geometry");
  if (g.oh != g.h + 2 * g.ph - 2 || g.ow != g.w + 2 * g.pw - 2 || g.oh <= 0 || g.ow <= 0)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "winograd_f32: output size does not match the geometry");
  if (!x_nchw || !u_hi || !out_nchw || !scratch || (split && !u_lo))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "winograd_f32: null operand");
  if (act < LSC_ACT_NONE || act > LSC_ACT_GELU) return set_error(LSC_ERROR_INVALID_ARGUMENT, "winograd_f32: bad activation");
  if (g.n == 0) return LSC_SUCCESS;
  const int64_t th = (g.oh + 1) / 2, tw = (g.ow + 1) / 2;
  const int64_t tiles = g.n * th * tw;
  if (16 * tiles * (cp > g.c_out ? cp : g.c_out) > INT32_MAX / 2 || g.n * th > 65535)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "winograd_f32: problem too large");
  float* vhi = scratch;
  float* vlo = split ? vhi + 16 * tiles * cp : nullptr;
  float* mm = vhi + 16 * tiles * cp * (split ? 2 : 1);
  const dim3 grid_in(static_cast<unsigned>((tw + kWT - 1) / kWT), static_cast<unsigned>(g.n * th),
                     static_cast<unsigned>((cp + kWC - 1) / kWC));
  winograd_input_kernel<<<grid_in, 256, 0, stream>>>(x_nchw, static_cast<int>(g.c), static_cast<int>(g.h),
                                                     static_cast<int>(g.w), static_cast<int>(g.ph),
                                                     static_cast<int>(g.pw), static_cast<int>(th),
                                                     static_cast<int>(tw), static_cast<int>(cp), tiles, vhi, vlo);
  LSC_CUDA_TRY(cudaGetLastError());
  lsc_status st = launch_gemm_tf32_batched(vhi, vlo, u_hi, u_lo, 16, tiles, g.c_out, cp, nullptr, LSC_ACT_NONE,
                                           mm, g.c_out, tiles * g.c_out, split, stream);
  if (st) return st;
  const dim3 grid_out(static_cast<unsigned>((tw + kWT - 1) / kWT), static_cast<unsigned>(g.n * th),
                      static_cast<unsigned>((g.c_out + kWC - 1) / kWC));
  winograd_output_kernel<<<grid_out, 256, 0, stream>>>(mm, tiles, static_cast<int>(g.c_out), static_cast<int>(th),
                                                       static_cast<int>(tw), static_cast<int>(g.oh),
                                                       static_cast<int>(g.ow), bias, act, out_nchw);
  LSC_CUDA_TRY(cudaGetLastError());
  return LSC_SUCCESS;
}

}  // namespace lsc
