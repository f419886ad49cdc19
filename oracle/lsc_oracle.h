/*
 * lsc_oracle.h -- CPU restatement of LightShip's dense-contraction math.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (lightship_b200/, include/)
 * links, loads or calls this library.  It is imported by tests/, by
 * __graft_entry__.smoke() and by bench.py's CPU-baseline leg, and only there as
 * the checker (or the timed CPU baseline), never as the thing that is measured
 * on the GPU or shipped.
 *
 * The reference (armsword/LightShip) is pure Rust and cannot be built in this
 * environment (no cargo/rustc, crates not vendored), so this file restates its
 * algorithms in C++.  Every function cites the reference file:line it follows;
 * paths are relative to the reference project root, with
 *   core/  = lightship-core/src/
 *   tests/ = lightship-core/tests/
 * Parity of this restatement is pinned against the reference's own known-answer
 * tests (tests/golden/ and tests/test_oracle_golden.py).
 *
 * Floating-point contract: compiled with -ffp-contract=off so that every
 * a*b+c stays two IEEE roundings, as in Rust (which never contracts).
 */
#ifndef LSC_ORACLE_H
#define LSC_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* rounding modes for the requantize step (R in the INT8 chain) */
#define ORC_ROUND_HALF_AWAY 0 /* Rust f32::round, core/cpu/quantized_ops.rs:45 */
#define ORC_ROUND_HALF_EVEN 1 /* round-half-even requantize variant              */

/* epilogue activations */
#define ORC_ACT_NONE 0
#define ORC_ACT_RELU 1  /* core/platform/simd.rs:552-556 */
#define ORC_ACT_RELU6 2 /* core/platform/simd.rs:558-562 */
#define ORC_ACT_SILU 3  /* core/operator/silu.rs:47-61   */
#define ORC_ACT_GELU 4  /* core/operator/gelu.rs:77-103  */

/* quantized dtypes understood by quantize_value / find_scale_zp */
#define ORC_QUINT8 0
#define ORC_QINT8 1
#define ORC_QINT32 2

const char* orc_version(void);

/* ---- FP32 GEMM family ---------------------------------------------------- */
/* gemm_scalar: C += A*B, sequential K sum (core/platform/simd.rs:588-598) */
void orc_gemm_scalar(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k);
/* gemm_neon loop nest: C += A*B with mc=64/kc=128 blocking and 16-column groups
 * (core/platform/simd.rs:1938-2052), including the m*n<512 simple path (:2055-2085) */
void orc_gemm_blocked(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k);
/* CpuBackend::execute_matmul: C = A*B (C zeroed), rows split in contiguous blocks
 * across `threads` (core/backend/cpu.rs:949-1063, core/cpu/thread_scheduler.rs:352-386) */
void orc_matmul(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k, int threads);
/* CpuBackend::execute_fullyconnected: Y[b,o] = sum_i X[b,i]*W[o,i] (core/backend/cpu.rs:1209-1290) */
void orc_fully_connected(const float* x, const float* w, float* y, int64_t batch, int64_t in_f,
                         int64_t out_f, int threads);

/* ---- Conv2d / BatchNorm / activations ----------------------------------- */
/* Conv2dConfig::output_shape (core/operator/convolution.rs:55-62). Returns -1 when the
 * unsigned arithmetic of the reference would underflow. */
int64_t orc_conv_out_dim(int64_t in, int64_t k, int64_t stride, int64_t pad, int64_t dil);
/* Conv2d::forward with the intended (kh,kw,c)-consistent K order: im2col + blocked GEMM,
 * NCHW input, OIHW filter, NCHW output, optional per-channel bias
 * (core/operator/convolution.rs:90-267).  bias may be NULL. */
void orc_conv2d_nchw(const float* x, const float* w, const float* bias, float* y, int64_t n,
                     int64_t c_in, int64_t h, int64_t wd, int64_t c_out, int64_t kh, int64_t kw,
                     int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh, int64_t dw,
                     int64_t groups, int threads);
/* Faithful restatement of the reference's im2col/filter pairing, including the K-order
 * mismatch (im2col (kh,kw,c) at convolution.rs:184-186 vs filter (c,kh,kw) at :252-254).
 * Diagnostic only: shows where the reference's own output departs from a convolution. */
void orc_conv2d_nchw_reference_korder(const float* x, const float* w, float* y, int64_t n,
                                      int64_t c_in, int64_t h, int64_t wd, int64_t c_out,
                                      int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                                      int64_t pw, int64_t dh, int64_t dw, int64_t groups);
/* BatchNorm::forward_inference per channel c over a [N,C,S] tensor with the channel-major
 * index fixed for N>1 (core/operator/batchnorm.rs:154-215).  Params may be NULL -> defaults
 * gamma=1, beta=0, mean=0, var=1 (batchnorm.rs:178-187). */
void orc_batchnorm_inference(const float* x, float* y, int64_t n, int64_t c, int64_t spatial,
                             const float* gamma, const float* beta, const float* mean,
                             const float* var, float eps);
/* BN fold (core/ir/optimizer.rs:727-731): w' = g/sqrt(v+eps)*w ; b' = g/sqrt(v+eps)*(b-mu)+beta.
 * w is [c_out, per_out]; bias may be NULL (treated as 0). */
void orc_bn_fold(const float* w, const float* bias, const float* gamma, const float* beta,
                 const float* mean, const float* var, float eps, int64_t c_out, int64_t per_out,
                 float* w_out, float* b_out);
float orc_act(float x, int act);
void orc_act_inplace(float* x, int64_t n, int act);
/* LayerNorm over the last axis of [rows, d]: (x - mean) / sqrt(var + eps), then * gamma[i],
   + beta[i] when given (core/operator/layernorm.rs:153-205). */
void orc_layernorm(const float* x, float* y, int64_t rows, int64_t d, const float* gamma,
                   const float* beta, float eps);
/* Softmax over the last axis of [rows, d] (core/operator/softmax.rs:106-146). */
void orc_softmax(const float* x, float* y, int64_t rows, int64_t d);

/* ---- quantization (core/quantization/helpers.rs, core/cpu/quantized_ops.rs) ---- */
float orc_round(float x, int rounding);
int32_t orc_quantize_value(float value, float scale, int32_t zero_point, int qdtype);
float orc_dequantize_value(int32_t q, float scale, int32_t zero_point);
/* find_scale_zp (helpers.rs:101-136): writes scale and zero point; returns 0 on empty input */
int orc_find_scale_zp(const float* data, int64_t n, int qdtype, int symmetric, float* scale,
                      int32_t* zero_point);
/* quantize_tensor / dequantize_tensor, per-tensor (helpers.rs:11-94); qdtype QINT8/QUINT8 */
void orc_quantize_tensor(const float* x, int64_t n, float scale, int32_t zp, int qdtype,
                         void* out);
void orc_dequantize_tensor(const void* q, int64_t n, float scale, int32_t zp, int qdtype,
                           float* out);
/* quantize_sym with a selectable rounding (quantized_ops.rs:43-48) */
void orc_quantize_sym(const float* x, int8_t* q, int64_t n, float scale, int rounding);
/* per-axis-0 symmetric weight quantization: s[c] from find_scale_zp over row c, then
 * quantize_value(w, s[c], 0, QInt8) (helpers.rs:101-155 applied per channel) */
void orc_quantize_weights_per_channel(const float* w, int64_t rows, int64_t cols, int8_t* q,
                                      float* scales);

/* ---- INT8 chain ----------------------------------------------------------- */
/* quantized_gemm_int8 as written: C[M,N] = A[M,K] * B[K,N] (NN), int32
 * (core/cpu/quantized_ops.rs:13-33) */
void orc_gemm_i8_nn(const int8_t* a, const int8_t* b, int32_t* c, int64_t m, int64_t n,
                    int64_t k, int threads);
/* the same sum with the weight stored [N,K] (FC / conv weight layout) */
void orc_gemm_i8_tn(const int8_t* a, const int8_t* w, int32_t* c, int64_t m, int64_t n,
                    int64_t k, int threads);
/* requantize/dequantize epilogue on an int32 accumulator tile [M,N]:
 *   acc += bias[n]; y = (float)acc * scale[n]; y = act(y);
 *   out_f32 = y; out_i8 = (i8)clamp(R(y / s_out), -128, 127)
 * (quantized_ops.rs:36-48, simd.rs:552-562, silu.rs:47-61).  Any output may be NULL. */
void orc_requant(const int32_t* acc, int64_t m, int64_t n, const int32_t* bias,
                 const float* scale, int act, float s_out, int rounding, int8_t* out_i8,
                 float* out_f32, int32_t* out_acc);
/* full chain with the [N,K] weight: GEMM + epilogue, threaded over M */
void orc_gemm_i8_chain(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                       const int32_t* bias, const float* scale, int act, float s_out,
                       int rounding, int8_t* out_i8, float* out_f32, int32_t* out_acc,
                       int threads);
/* INT8 direct convolution, NHWC activations [N,H,W,C], weight [Cout,KH,KW,Cin/groups],
 * followed by the same epilogue; output NHWC [N,OH,OW,Cout]. */
void orc_conv2d_i8_nhwc_chain(const int8_t* x, const int8_t* w, int64_t n, int64_t h,
                              int64_t wd, int64_t c_in, int64_t c_out, int64_t kh, int64_t kw,
                              int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh,
                              int64_t dw, int64_t groups, const int32_t* bias,
                              const float* scale, int act, float s_out, int rounding,
                              int8_t* out_i8, float* out_f32, int32_t* out_acc, int threads);

/* The same with a residual added before the activation: y = dequant(acc) + (f32)r * r_scale,
 * r int8 NHWC shaped like the output (a ResNet BasicBlock's Add + ReLU after its second conv;
 * dequantize_value with zero point 0, helpers.rs:158-160). */
void orc_conv2d_i8_nhwc_chain_res(const int8_t* x, const int8_t* w, int64_t n, int64_t h,
                                  int64_t wd, int64_t c_in, int64_t c_out, int64_t kh, int64_t kw,
                                  int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh,
                                  int64_t dw, const int32_t* bias, const float* scale, int act,
                                  float s_out, int rounding, const int8_t* residual,
                                  float r_scale, int8_t* out_i8, float* out_f32, int32_t* out_acc,
                                  int threads);
/* f32 NCHW -> int8 NHWC with channels padded to cp (quantize_value, helpers.rs:139-155, with R) */
void orc_quantize_nchw_to_nhwc(const float* x, int8_t* y, int64_t n, int64_t c, int64_t hw,
                               int64_t cp, float scale, int rounding);
/* MaxPool2d on int8 NHWC codes, padding taps skipped (operator/pooling.rs:383-455) */
void orc_maxpool_i8_nhwc(const int8_t* x, int8_t* y, int64_t n, int64_t h, int64_t w, int64_t c,
                         int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw);
/* GlobalAvgPool2d on int8 NHWC (operator/pooling.rs:457-530): y = ((f32)sum_q * s_in) / (H*W),
 * then requantized with s_out (y_i8) and/or kept (y_f32) */
void orc_avgpool_i8_nhwc(const int8_t* x, int64_t n, int64_t hw, int64_t c, float s_in,
                         float s_out, int rounding, int8_t* y_i8, float* y_f32);

#ifdef __cplusplus
}
#endif
#endif
