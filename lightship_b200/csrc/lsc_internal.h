// lsc_internal.h -- shared host-side declarations of the CUDA backend library.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "lightship_cuda.h"

namespace lsc {

// Records a message for lsc_last_error() on this thread and returns `code`.
lsc_status set_error(lsc_status code, const char* fmt, ...);
// Maps a CUDA runtime error to LSC_ERROR_DEVICE_ERROR (or OUT_OF_MEMORY) with a message.
lsc_status cuda_error(cudaError_t e, const char* what);

#define LSC_CUDA_TRY(expr)                                 \
  do {                                                     \
    cudaError_t _e = (expr);                               \
    if (_e != cudaSuccess) return ::lsc::cuda_error(_e, #expr); \
  } while (0)

// Per-device facts and the device-resident error word, set up once per device.
struct DeviceState {
  int device = -1;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  size_t smem_optin = 0;
  size_t total_memory = 0;
  uint32_t* err_word = nullptr;  // device address of the sticky error word
  bool overlap_launches = true;  // dependent launches (LSC_OVERLAP_LAUNCHES=0 turns them off)
};

// Launches `kernel` with programmatic stream serialization when `overlap` is set: its CTAs may
// be scheduled, and run their prologue, while the previous kernel on the stream is finishing.
// Every kernel launched this way calls griddep_wait() before it reads what an earlier kernel
// wrote or writes what an earlier kernel may still read.  Graph capture keeps the relation.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_dependent(bool overlap, void (*kernel)(KArgs...), dim3 grid, dim3 block,
                                    size_t smem, cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = overlap ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

#ifdef __CUDACC__
// Device side of a dependent launch.  griddep_wait(): blocks the calling thread until the
// kernels this grid depends on have completed and their memory is visible (returns at once
// when the launch had no such dependency).  griddep_launch_dependents(): this CTA allows the
// next dependent kernel to be scheduled; it starts once every CTA has said so or exited.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
#endif

// State of the calling thread's current device; nullptr (with the error set) on failure.
DeviceState* current_device_state();
DeviceState* device_state(int device);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda needed).
// 2-D tensor: `inner` contiguous elements per row, `outer` rows, `row_stride_bytes` apart.
lsc_status encode_tmap_2d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                          uint64_t inner, uint64_t outer, uint64_t row_stride_bytes,
                          uint32_t box_inner, uint32_t box_outer, CUtensorMapSwizzle swizzle);
lsc_status encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                          const uint64_t dims[3], const uint64_t strides_bytes[2],
                          const uint32_t box[3], const uint32_t elem_strides[3],
                          CUtensorMapSwizzle swizzle);
lsc_status encode_tmap_4d(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                          const uint64_t dims[4], const uint64_t strides_bytes[3],
                          const uint32_t box[4], const uint32_t elem_strides[4],
                          CUtensorMapSwizzle swizzle);

// 4-D NHWC tensor map in im2col mode (cuTensorMapEncodeIm2col).
lsc_status encode_tmap_im2col(CUtensorMap* map, CUtensorMapDataType dtype, const void* base,
                              const uint64_t dims[4], const uint64_t strides_bytes[3],
                              const int lower[2], const int upper[2], uint32_t channels_per_pixel,
                              uint32_t pixels_per_column, const uint32_t elem_strides[4],
                              CUtensorMapSwizzle swizzle);

// Convolution geometry for the NHWC INT8 implicit GEMM.
struct ConvGeometry {
  int64_t n, h, w, c;       // input NHWC; c = channels as stored (multiple of 16)
  int64_t c_out;
  int64_t kh, kw;
  int64_t sh, sw, ph, pw, dh, dw;
  int64_t oh, ow;
  int64_t ph_b, pw_r;       // bottom / right padding (= ph / pw unless asymmetric; < 0 crops)
};

// INT8 NHWC convolution as an implicit GEMM (contraction_i8.cu): x [N,H,W,C] int8,
// w [Cout, KH*KW*C] int8 (K ordered kh, kw, c), outputs NHWC [N,OH,OW,Cout].  `residual`
// (optional, int8 NHWC like the outputs) is added as (f32)r * res_scale before the activation.
lsc_status launch_conv_i8(const int8_t* x, const int8_t* w, const ConvGeometry& g,
                          const int32_t* bias, const float* scale, float s_out, int act,
                          int rounding, int8_t* out_i8, float* out_f32, int32_t* out_i32,
                          const int8_t* residual, float res_scale, cudaStream_t stream);
// A pixel-grouped ReLU convolution (grouped geometry g: the NHWC input viewed with `group`
// pixels per row group, filter [256 = group * Cout, KH, KWg, C]) with the 3x3 / 2 max pool of
// padding 1 over its ungrouped output fused in: out_pool is [N, OH / 2, OW * group / 2, Cout]
// int8 (the CNN stem's convolution and max pool in one launch; contraction_i8.cu).
lsc_status launch_conv_pool_i8(const int8_t* x, const int8_t* w, const ConvGeometry& g, int group,
                               const int32_t* bias, const float* scale, float s_out, int act, int rounding,
                               int8_t* out_pool, cudaStream_t stream);
// The ResNet stem in one launch (stem_i8.cu): f32 NCHW x [n, 3, 224, 224] quantized with s_in
// (rounding_in), the 7x7 / 2 convolution of padding 3 to 64 channels with the INT8 chain's
// epilogue (bias, per-channel scale, ReLU, requantization by s_out), then the 3x3 / 2 max pool
// of padding 1: out [n, 56, 56, 64] int8 NHWC.  The filter is w_img, kStemFilterBytes made by
// stem_filter_image.  Bit-exact with the separate launches when every scale[c] > 0 and
// |bias[c]| < 2^30 (the caller checks).
constexpr int64_t kStemFilterBytes = 12288;
lsc_status launch_stem_conv_pool_i8(const float* x, int64_t n, const int8_t* w_img, const int32_t* bias,
                                    const float* scale, float s_in, int rounding_in, float s_out, int rounding,
                                    int8_t* out, cudaStream_t stream);
// The stem kernel's filter image from the space-to-depth filter [64][4][4][16] (host bytes).
void stem_filter_image(const int8_t* w_s2d, int8_t* img);

// INT8 GEMM + requant/dequant epilogue (contraction_i8.cu).  ldo = row stride of the outputs in
// elements.  Validates its arguments.
// Optional extras of the GEMM chain: an f16 copy of the (activated) f32 result and an f32
// residual [M, ldo] added before the activation.
struct GemmExtras {
  void* out_f16 = nullptr;
  const float* res_f32 = nullptr;
};
lsc_status launch_gemm_i8(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                          const int32_t* bias, const float* scale, float s_out, int act,
                          int rounding, int8_t* out_i8, float* out_f32, int32_t* out_i32,
                          int64_t ldo, cudaStream_t stream, const GemmExtras* extras = nullptr);

// FP32 contractions as split-TF32 (contraction_tf32.cu).  GEMM: A [M,K] and B [N,K] K-major
// (hi and lo parts; lo unused when split == false), K a multiple of 4, output row-major with
// stride ldo.  Convolution: NHWC hi/lo input with g.c stored channels (multiple of 4),
// weights [Cout, KH*KW*C], output NCHW.
// Small products with a long K (fewer output tiles than half the SMs) split K over more CTAs
// when the caller passes `ksplit_ws`, device scratch of the floats tf32_gemm_ksplit_floats /
// tf32_conv_ksplit_floats return (0: no split for that shape); the partial sums are added in a
// fixed order by a second launch.
int64_t tf32_gemm_ksplit_floats(int64_t m, int64_t n, int64_t k);
int64_t tf32_conv_ksplit_floats(const ConvGeometry& g);
lsc_status launch_gemm_tf32(const float* a_hi, const float* a_lo, const float* b_hi,
                            const float* b_lo, int64_t m, int64_t n, int64_t k,
                            const float* bias, int act, float* out, int64_t ldo, bool split,
                            cudaStream_t stream, float* ksplit_ws = nullptr, int64_t ksplit_ws_floats = 0);
lsc_status launch_conv_tf32(const float* x_hi, const float* x_lo, const float* w_hi,
                            const float* w_lo, const ConvGeometry& g, const float* bias, int act,
                            float* out_nchw, bool split, cudaStream_t stream, float* ksplit_ws = nullptr,
                            int64_t ksplit_ws_floats = 0);
// `batches` GEMMs in one launch: batch b's A is rows [b*m, (b+1)*m) of a_hi/a_lo, its B rows
// [b*n, (b+1)*n) of b_hi/b_lo, its output out + b * out_batch_stride.
lsc_status launch_gemm_tf32_batched(const float* a_hi, const float* a_lo, const float* b_hi,
                                    const float* b_lo, int64_t batches, int64_t m, int64_t n, int64_t k,
                                    const float* bias, int act, float* out, int64_t ldo,
                                    int64_t out_batch_stride, bool split, cudaStream_t stream,
                                    float* ksplit_ws = nullptr, int64_t ksplit_ws_floats = 0);
// FP32 3x3 stride-1 convolution as Winograd F(2x2, 3x3) (winograd_f32.cu): NCHW input with
// g.c channels, transformed filter u [16][Cout][cp] (hi/lo), NCHW output; `scratch` holds
// winograd_f32_scratch_floats(g, cp, split) floats.
int64_t winograd_f32_scratch_floats(const ConvGeometry& g, int64_t cp, bool split);
lsc_status launch_conv_winograd_f32(const float* x_nchw, const float* u_hi, const float* u_lo,
                                    const ConvGeometry& g, int64_t cp, const float* bias, int act,
                                    float* out_nchw, float* scratch, bool split, cudaStream_t stream);
// Operand preparation (tf32_prep.cu): split into hi/lo parts with padding / transposition.
lsc_status prep_split_rows(const float* x, int64_t rows, int64_t cols, int64_t ld, float* hi,
                           float* lo, cudaStream_t st);
lsc_status prep_split_transpose(const float* x, int64_t k, int64_t n, int64_t ldk, float* hi,
                                float* lo, cudaStream_t st);
lsc_status prep_split_nchw_to_nhwc(const float* x, int64_t n, int64_t c, int64_t hw, int64_t cp,
                                   float* hi, float* lo, cudaStream_t st);
// Elementwise FP32 operators (elementwise.cu).
lsc_status launch_batchnorm_f32(const float* x, float* y, int64_t n, int64_t c, int64_t spatial,
                                const float* gamma, const float* beta, const float* mean,
                                const float* inv_std, int act, cudaStream_t st);
lsc_status launch_activation_f32(const float* x, float* y, int64_t n, int act, cudaStream_t st);
lsc_status launch_add_f32(const float* a, const float* b, float* y, int64_t n, int act,
                          cudaStream_t st);

// INT8 NHWC glue (pool.cu).
lsc_status launch_quantize_nchw_to_nhwc_i8(const float* x, int8_t* y, int64_t n, int64_t c,
                                           int64_t hw, int64_t cp, float scale, int rounding,
                                           cudaStream_t st);
// Row-wise LayerNorm / Softmax over the last axis of [rows, d], f32 or f16 storage (norm.cu).
// LayerNorm writes int8 to q (R(y / q_scale), saturated) instead of y when q is non-null.
lsc_status launch_layernorm(const void* x, void* y, int32_t dtype, int64_t rows, int64_t d, const float* gamma,
                            const float* beta, float eps, cudaStream_t st, int8_t* q = nullptr,
                            float q_scale = 0.0f, int rounding = LSC_ROUND_HALF_AWAY);
// RN(1 / s) when s and 1/s are normal floats, else 0 (pool.cu).
float reciprocal_or_zero(float s);
// y[b][h][c][r] = x[b][h + h0][r][c], f16 (contraction_f16.cu).
lsc_status launch_transpose_heads_f16(const void* x, void* y, int64_t xb, int64_t xh, int64_t xr, int64_t h0,
                                      int64_t batch, int64_t heads, int64_t rows, int64_t cols, cudaStream_t stream);
// Fused attention over a [batch, seq, 3, heads, 64] f16 QKV projection (attention_f16.cu).
lsc_status launch_attention_f16(const void* qkv, int64_t batch, int64_t seq, int64_t heads, float alpha,
                                float* out_f32, int8_t* out_i8, float s_out, int rounding, cudaStream_t stream);
lsc_status launch_softmax(const void* x, void* y, int32_t dtype, int64_t rows, int64_t d, cudaStream_t st);

lsc_status launch_quantize_nchw_to_s2d_i8(const float* x, int8_t* y, int64_t n, int64_t c, int64_t h,
                                          int64_t w, int64_t ph, int64_t pw, int64_t ph_end, int64_t pw_end,
                                          int64_t blk, int64_t cp, float scale, int rounding, cudaStream_t st);
lsc_status launch_maxpool_i8(const int8_t* x, int8_t* y, int64_t n, int64_t h, int64_t w, int64_t c,
                             int64_t oh, int64_t ow, int kh, int kw, int sh, int sw, int ph, int pw,
                             cudaStream_t st);
lsc_status launch_maxpool_f32(const float* x, float* y, int64_t n, int64_t c, int64_t h, int64_t w, int64_t oh,
                              int64_t ow, int kh, int kw, int sh, int sw, int ph, int pw, cudaStream_t st);
lsc_status launch_avgpool_f32(const float* x, float* y, int64_t n, int64_t c, int64_t hw, cudaStream_t st);
lsc_status launch_avgpool_i8(const int8_t* x, int64_t n, int64_t hw, int64_t c, float s_in, float s_out,
                             int rounding, int8_t* y_i8, float* y_f32, cudaStream_t st);

// Quantization kernels (quant.cu).  `scales` == nullptr selects the per-tensor form with
// scale0/zp0; otherwise channel c = (i / inner) % channels.
lsc_status launch_quantize(const float* x, void* out, int64_t n, int qdtype, const float* scales,
                           const int32_t* zps, float scale0, int32_t zp0, int32_t channels,
                           int64_t inner, int rounding, cudaStream_t st);
lsc_status launch_dequantize(const void* q, int qdtype, float* out, int64_t n, const float* scales,
                             const int32_t* zps, float scale0, int32_t zp0, int32_t channels,
                             int64_t inner, cudaStream_t st);
constexpr uint64_t kFindScaleZpWorkspace = 16;
lsc_status launch_find_scale_zp(const float* x, int64_t n, int qdtype, int symmetric,
                                void* workspace, uint64_t workspace_bytes, float* scale_out,
                                int32_t* zp_out, cudaStream_t st);

}  // namespace lsc
