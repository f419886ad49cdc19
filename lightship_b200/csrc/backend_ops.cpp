// backend_ops.cpp -- compile/execute of each operator the CUDA backend runs.
//
// Compile-time work (weights only): transposes to K-major, K padding to the TMA granule,
// per-channel symmetric INT8 weight quantization (find_scale_zp + quantize_value per output
// channel, quantization/helpers.rs:101-155), s[n] = s_a * s_w[n] (cpu/quantized_ops.rs:11).
// All host arithmetic here is compiled with -ffp-contract=off so it rounds like the
// reference's Rust code.
#include <math.h>
#include <string.h>

#include <vector>

#include "backend_ops.h"

namespace lsc {

uint32_t supported_ops_mask() {
  return (1u << LSC_OP_QGEMM) | (1u << LSC_OP_FULLY_CONNECTED) | (1u << LSC_OP_QUANTIZE) |
         (1u << LSC_OP_DEQUANTIZE) | (1u << LSC_OP_CONV2D) | (1u << LSC_OP_MATMUL) |
         (1u << LSC_OP_BATCHNORM) | (1u << LSC_OP_RELU) | (1u << LSC_OP_RELU6) |
         (1u << LSC_OP_SILU) | (1u << LSC_OP_MAXPOOL2D) | (1u << LSC_OP_GLOBAL_AVGPOOL2D) |
         (1u << LSC_OP_GELU) | (1u << LSC_OP_LAYERNORM) | (1u << LSC_OP_SOFTMAX) | (1u << LSC_OP_ADD);
}

namespace {

const char* tname(const lsc_tensor& t) { return t.name ? t.name : "?"; }

int act_of(const lsc_op_desc& d) {
  switch (d.fusion) {
    case LSC_FUSION_CONV_RELU:
    case LSC_FUSION_BATCHNORM_RELU:
    case LSC_FUSION_ADD_RELU:
    case LSC_FUSION_MUL_RELU: return LSC_ACT_RELU;
    case LSC_FUSION_CONV_RELU6: return LSC_ACT_RELU6;
    default: return d.activation;
  }
}

// Rust `f32 as i32` (saturating, NaN -> 0).
int32_t sat_i32(float v) {
  if (v != v) return 0;
  if (v >= 2147483648.0f) return INT32_MAX;
  if (v <= -2147483648.0f) return INT32_MIN;
  return static_cast<int32_t>(v);
}

// Symmetric per-row INT8 quantization of an f32 [rows, cols] weight: s = absmax/127
// (1.0 for an all-zero row), q = clamp(round_half_away(w / s), -128, 127).
void quantize_rows_sym(const float* w, int64_t rows, int64_t cols, int8_t* q, float* s) {
  for (int64_t r = 0; r < rows; ++r) {
    float mn = INFINITY, mx = -INFINITY;
    for (int64_t c = 0; c < cols; ++c) {
      mn = fminf(mn, w[r * cols + c]);
      mx = fmaxf(mx, w[r * cols + c]);
    }
    const float am = fmaxf(fabsf(mx), fabsf(mn));
    const float sc = am > 0.0f ? am / 127.0f : 1.0f;
    s[r] = sc;
    for (int64_t c = 0; c < cols; ++c) {
      int32_t v = sat_i32(roundf(w[r * cols + c] / sc));
      v = v < -128 ? -128 : (v > 127 ? 127 : v);
      q[r * cols + c] = static_cast<int8_t>(v);
    }
  }
}

lsc_status own_upload(lsc_op* op, const void* host, int64_t bytes, void** dptr) {
  lsc_status st = upload(op->be, host, bytes, dptr);
  if (st == LSC_SUCCESS) op->owned.push_back(*dptr);
  return st;
}

// ---------------------------------------------------------------- INT8 contraction
// QGEMM: in[0] A [M,K] int8 (quant.scale = s_a), in[1] B [K,N] (quantized_gemm_int8's NN
// layout), in[2] optional bias [N] i32.  FULLY_CONNECTED with int8 input: in[1] W [N,K].
lsc_status compile_qgemm(lsc_op* op, const lsc_tensor* in, int n_in, const lsc_tensor* out,
                         int n_out, bool weight_nk) {
  if (n_in < 2 || n_out < 1)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantized GEMM needs >= 2 inputs and >= 1 output");
  const lsc_tensor& a = in[0];
  const lsc_tensor& w = in[1];
  if (!is_int8(a.dtype))
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "quantized GEMM: input '%s' must be int8", tname(a));
  if (a.ndim != 2 || w.ndim != 2)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantized GEMM requires 2D matrices");
  const int64_t k = a.shape[1];
  const int64_t wk = weight_nk ? w.shape[1] : w.shape[0];
  const int64_t n = weight_nk ? w.shape[0] : w.shape[1];
  if (wk != k)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "Matrix dimension mismatch: A_cols=%lld != B_rows=%lld",
                     (long long)k, (long long)wk);
  if (k <= 0 || n <= 0) return set_error(LSC_ERROR_SHAPE_MISMATCH, "quantized GEMM: empty K or N");
  const float s_a = a.quant.count > 0 && a.quant.scale ? a.quant.scale[0] : 1.0f;

  // weights -> int8 [N, K] plus per-channel s_w
  std::vector<int8_t> wq(static_cast<size_t>(n * k));
  std::vector<float> sw(static_cast<size_t>(n));
  std::vector<uint8_t> raw;
  if (is_int8(w.dtype)) {
    lsc_status st = read_tensor_bytes(w, n * k, raw);
    if (st) return st;
    const int8_t* src = reinterpret_cast<const int8_t*>(raw.data());
    for (int64_t i = 0; i < n; ++i)
      for (int64_t j = 0; j < k; ++j)
        wq[i * k + j] = weight_nk ? src[i * k + j] : src[j * n + i];
    if (w.quant.count == 1 && w.quant.scale) {
      for (int64_t i = 0; i < n; ++i) sw[i] = w.quant.scale[0];
    } else if (w.quant.count == n && w.quant.scale) {
      for (int64_t i = 0; i < n; ++i) sw[i] = w.quant.scale[i];
    } else if (w.quant.count == 0) {
      for (int64_t i = 0; i < n; ++i) sw[i] = 1.0f;
    } else {
      return set_error(LSC_ERROR_INVALID_ARGUMENT, "weight '%s': %d scales for %lld channels",
                       tname(w), w.quant.count, (long long)n);
    }
    if (w.quant.zero_point)
      for (int i = 0; i < w.quant.count; ++i)
        if (w.quant.zero_point[i] != 0)
          return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "weight '%s': only symmetric (zp = 0) INT8 weights", tname(w));
  } else if (w.dtype == LSC_DTYPE_F32) {
    lsc_status st = read_tensor_bytes(w, n * k * 4, raw);
    if (st) return st;
    const float* src = reinterpret_cast<const float*>(raw.data());
    std::vector<float> wt(static_cast<size_t>(n * k));
    for (int64_t i = 0; i < n; ++i)
      for (int64_t j = 0; j < k; ++j) wt[i * k + j] = weight_nk ? src[i * k + j] : src[j * n + i];
    quantize_rows_sym(wt.data(), n, k, wq.data(), sw.data());
  } else {
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "weight '%s': dtype %d", tname(w), w.dtype);
  }

  // K padded to the 16-byte TMA granule; padding columns are zero
  const int64_t kp = (k + 15) / 16 * 16;
  std::vector<int8_t> wp(static_cast<size_t>(n * kp), 0);
  for (int64_t i = 0; i < n; ++i) memcpy(&wp[i * kp], &wq[i * k], static_cast<size_t>(k));
  std::vector<float> scale(static_cast<size_t>(n));
  for (int64_t i = 0; i < n; ++i) scale[i] = s_a * sw[i];

  lsc_status st = own_upload(op, wp.data(), n * kp, &op->w);
  if (st) return st;
  void* p = nullptr;
  if ((st = own_upload(op, scale.data(), n * 4, &p))) return st;
  op->scale = static_cast<float*>(p);
  if (n_in >= 3 && in[2].data) {
    const lsc_tensor& b = in[2];
    if (b.dtype != LSC_DTYPE_I32 && b.dtype != LSC_DTYPE_QINT32 && b.dtype != LSC_DTYPE_F32)
      return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "bias '%s' must be int32 or f32", tname(b));
    if (numel(b) != n) return set_error(LSC_ERROR_SHAPE_MISMATCH, "bias '%s' must have %lld entries", tname(b), (long long)n);
    if ((st = read_tensor_bytes(b, n * 4, raw))) return st;
    if (b.dtype == LSC_DTYPE_F32) {
      // f32 bias -> int32 in accumulator units: quantize_value(b, s_a * s_w[n], 0, QInt32)
      const float* bf = reinterpret_cast<const float*>(raw.data());
      std::vector<int32_t> bi(static_cast<size_t>(n));
      for (int64_t i = 0; i < n; ++i) bi[i] = sat_i32(roundf(bf[i] / scale[i]));
      if ((st = own_upload(op, bi.data(), n * 4, &p))) return st;
    } else if ((st = own_upload(op, raw.data(), n * 4, &p))) {
      return st;
    }
    op->bias_i32 = static_cast<int32_t*>(p);
  }
  for (int i = 0; i < n_out; ++i) {
    const int32_t dt = out[i].dtype;
    if (!(is_int8(dt) || dt == LSC_DTYPE_F32 || dt == LSC_DTYPE_F16 || dt == LSC_DTYPE_I32 || dt == LSC_DTYPE_QINT32))
      return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "output '%s': dtype %d", tname(out[i]), dt);
    if (is_int8(dt)) {
      float so = op->desc.output_scale;
      if (!(so > 0.0f) && out[i].quant.count > 0 && out[i].quant.scale) so = out[i].quant.scale[0];
      if (!(so > 0.0f))
        return set_error(LSC_ERROR_INVALID_ARGUMENT, "int8 output '%s' needs an output scale", tname(out[i]));
      op->s_out = so;
    }
  }
  op->kind = OpKind::kQGemm;
  op->n = n;
  op->k = k;
  op->kp = kp;
  op->act = act_of(op->desc);
  return LSC_SUCCESS;
}

lsc_status execute_qgemm(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                         int n_out, Staging& s) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantized GEMM: missing tensors");
  const lsc_tensor& a = in[0];
  if (!is_int8(a.dtype)) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "input '%s' must be int8", tname(a));
  if (a.ndim != 2 || a.shape[1] != op->k)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "input '%s' must be [M, %lld]", tname(a), (long long)op->k);
  const int64_t m = a.shape[0], n = op->n, k = op->k, kp = op->kp;
  const void* ad = nullptr;
  if (kp == k) {
    lsc_status st = s.input(a, m * k, &ad);
    if (st) return st;
  } else {
    if (m * k > 0 && !a.data) return set_error(LSC_ERROR_INVALID_ARGUMENT, "input '%s' has no data", tname(a));
    void* pad = s.scratch(m * kp);
    if (!pad) return LSC_ERROR_OUT_OF_MEMORY;
    LSC_CUDA_TRY(cudaMemsetAsync(pad, 0, static_cast<size_t>(m * kp), s.st));
    if (m > 0)
      LSC_CUDA_TRY(cudaMemcpy2DAsync(pad, static_cast<size_t>(kp), a.data, static_cast<size_t>(k),
                                     static_cast<size_t>(k), static_cast<size_t>(m),
                                     a.location == LSC_MEM_DEVICE ? cudaMemcpyDeviceToDevice
                                                                  : cudaMemcpyHostToDevice,
                                     s.st));
    if (a.location != LSC_MEM_DEVICE) s.touched_host = true;
    ad = pad;
  }
  int8_t* o_i8 = nullptr;
  float* o_f32 = nullptr;
  int32_t* o_i32 = nullptr;
  GemmExtras ex;
  float s_out = op->s_out;
  for (int i = 0; i < n_out; ++i) {
    lsc_tensor& t = out[i];
    const int64_t es = dtype_size(t.dtype);
    void* d = nullptr;
    lsc_status st = s.output(t, m * n * es, &d);
    if (st) return st;
    if (is_int8(t.dtype)) {
      o_i8 = static_cast<int8_t*>(d);
      // a calibrated output scale carried by the output tensor overrides the compiled one
      if (t.quant.count > 0 && t.quant.scale && t.quant.scale[0] > 0.0f) s_out = t.quant.scale[0];
    } else if (t.dtype == LSC_DTYPE_F32) {
      o_f32 = static_cast<float*>(d);
    } else if (t.dtype == LSC_DTYPE_F16) {
      ex.out_f16 = d;
    } else {
      o_i32 = static_cast<int32_t*>(d);
    }
    set_shape(t, {m, n});
  }
  // optional f32 residual (execute-time input 1), [M, N], added before the activation
  if (n_in >= 2 && in[1].data) {
    const lsc_tensor& r = in[1];
    if (r.dtype != LSC_DTYPE_F32) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "GEMM residual must be f32");
    if (numel(r) != m * n) return set_error(LSC_ERROR_SHAPE_MISMATCH, "GEMM residual '%s' must be [M, N]", tname(r));
    const void* rd = nullptr;
    lsc_status st = s.input(r, m * n * 4, &rd);
    if (st) return st;
    ex.res_f32 = static_cast<const float*>(rd);
  }
  if (m == 0) return LSC_SUCCESS;
  return launch_gemm_i8(static_cast<const int8_t*>(ad), static_cast<const int8_t*>(op->w), m, n, kp,
                        op->bias_i32, op->scale, s_out, op->act, op->rounding, o_i8, o_f32,
                        o_i32, n, s.st, &ex);
}

// ---------------------------------------------------------------- quantize / dequantize
lsc_status take_qparams(lsc_op* op, const lsc_tensor& t) {
  const lsc_quant& q = t.quant;
  if (q.count <= 1) {
    op->q_channels = 0;
    op->q_scale0 = q.count == 1 && q.scale ? q.scale[0] : 1.0f;
    op->q_zp0 = q.count == 1 && q.zero_point ? q.zero_point[0] : 0;
    return LSC_SUCCESS;
  }
  if (!q.scale) return set_error(LSC_ERROR_INVALID_ARGUMENT, "tensor '%s': per-channel scales missing", tname(t));
  op->q_channels = q.count;
  op->q_axis = t.layout == LSC_LAYOUT_NHWC ? t.ndim - 1 : (t.ndim >= 2 ? 1 : 0);
  if (op->q_axis < 0 || op->q_axis >= t.ndim || t.shape[op->q_axis] != q.count)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "tensor '%s': %d scales do not match its channel axis",
                     tname(t), q.count);
  void* p = nullptr;
  lsc_status st = own_upload(op, q.scale, q.count * 4, &p);
  if (st) return st;
  op->q_scales = static_cast<float*>(p);
  if (q.zero_point) {
    if ((st = own_upload(op, q.zero_point, q.count * 4, &p))) return st;
    op->q_zps = static_cast<int32_t*>(p);
  }
  return LSC_SUCCESS;
}

int64_t inner_of(const lsc_tensor& t, int axis) {
  int64_t inner = 1;
  for (int i = axis + 1; i < t.ndim; ++i) inner *= t.shape[i];
  return inner;
}

lsc_status execute_quant(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                         int n_out, Staging& s, bool quantize) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "quantize/dequantize: missing tensors");
  const lsc_tensor& x = in[0];
  lsc_tensor& y = out[0];
  const int64_t n = numel(x);
  if (n < 0) return set_error(LSC_ERROR_SHAPE_MISMATCH, "tensor '%s': bad shape", tname(x));
  const int32_t in_dt = quantize ? LSC_DTYPE_F32 : op->qdtype;
  const int32_t out_dt = quantize ? op->qdtype : LSC_DTYPE_F32;
  if (x.dtype != in_dt && !(is_int8(x.dtype) && is_int8(in_dt)))
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "input '%s': dtype %d, expected %d", tname(x), x.dtype, in_dt);
  const void* xd = nullptr;
  void* yd = nullptr;
  lsc_status st = s.input(x, n * dtype_size(in_dt), &xd);
  if (st) return st;
  if (quantize && op->kp > 0) {
    // f32 NCHW -> int8 NHWC with the channels padded to op->kp (a quantized CNN's input)
    if (x.ndim != 4) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Quantize to NHWC needs a 4D NCHW input");
    const int64_t nb = x.shape[0], c = x.shape[1], hw = x.shape[2] * x.shape[3];
    if (op->sh > 1) {
      const int64_t b = op->sh, hs = (x.shape[2] + op->ph + op->ph_end) / b;
      const int64_t ws = (x.shape[3] + op->pw + op->pw_end) / b;
      if ((st = s.output(y, nb * hs * ws * op->kp, &yd))) return st;
      set_shape(y, {nb, hs, ws, op->kp});
      return launch_quantize_nchw_to_s2d_i8(static_cast<const float*>(xd), static_cast<int8_t*>(yd), nb, c,
                                            x.shape[2], x.shape[3], op->ph, op->pw, op->ph_end, op->pw_end, b,
                                            op->kp, op->q_scale0, op->rounding, s.st);
    }
    if (c > op->kp) return set_error(LSC_ERROR_SHAPE_MISMATCH, "Quantize to NHWC: %lld channels exceed %lld", (long long)c, (long long)op->kp);
    if ((st = s.output(y, nb * hw * op->kp, &yd))) return st;
    set_shape(y, {nb, x.shape[2], x.shape[3], op->kp});
    return launch_quantize_nchw_to_nhwc_i8(static_cast<const float*>(xd), static_cast<int8_t*>(yd), nb, c, hw,
                                           op->kp, op->q_scale0, op->rounding, s.st);
  }
  if ((st = s.output(y, n * dtype_size(out_dt), &yd))) return st;
  y.ndim = x.ndim;
  for (int i = 0; i < x.ndim; ++i) y.shape[i] = x.shape[i];
  const int64_t inner = op->q_channels ? inner_of(x, op->q_axis) : 1;
  if (op->q_channels && (x.ndim <= op->q_axis || x.shape[op->q_axis] != op->q_channels))
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "input '%s': channel axis does not hold %d channels",
                     tname(x), op->q_channels);
  if (quantize)
    return launch_quantize(static_cast<const float*>(xd), yd, n, op->qdtype,
                           op->q_channels ? op->q_scales : nullptr, op->q_zps, op->q_scale0, op->q_zp0,
                           op->q_channels ? op->q_channels : 1, inner, op->rounding, s.st);
  return launch_dequantize(xd, op->qdtype, static_cast<float*>(yd), n,
                           op->q_channels ? op->q_scales : nullptr, op->q_zps, op->q_scale0, op->q_zp0,
                           op->q_channels ? op->q_channels : 1, inner, s.st);
}

}  // namespace

lsc_status compile_op(lsc_backend* be, lsc_op* op, const lsc_tensor* in, int n_in,
                      const lsc_tensor* out, int n_out) {
  (void)be;
  switch (op->desc.op_type) {
    case LSC_OP_QGEMM:
      return compile_qgemm(op, in, n_in, out, n_out, false);
    case LSC_OP_FULLY_CONNECTED:
      if (n_in >= 1 && is_int8(in[0].dtype)) return compile_qgemm(op, in, n_in, out, n_out, true);
      if (n_in >= 1 && in[0].dtype == LSC_DTYPE_F32) return compile_fc_f32(op, in, n_in, n_out);
      break;
    case LSC_OP_CONV2D:
      if (n_in >= 1 && (is_int8(in[0].dtype) || in[0].dtype == LSC_DTYPE_F32))
        return compile_conv(op, in, n_in, out, n_out);
      break;
    case LSC_OP_MATMUL:
      if (n_in >= 1 && in[0].dtype == LSC_DTYPE_F32) return compile_matmul_f32(op, in, n_in, n_out);
      break;
    case LSC_OP_BATCHNORM:
      if (n_in >= 1 && in[0].dtype == LSC_DTYPE_F32) return compile_batchnorm(op, in, n_in, n_out);
      break;
    case LSC_OP_MAXPOOL2D: return compile_pool(op, in, n_in, n_out, false);
    case LSC_OP_GLOBAL_AVGPOOL2D: return compile_pool(op, in, n_in, n_out, true);
    case LSC_OP_RELU: return compile_activation(op, in, n_in, n_out, LSC_ACT_RELU);
    case LSC_OP_RELU6: return compile_activation(op, in, n_in, n_out, LSC_ACT_RELU6);
    case LSC_OP_SILU: return compile_activation(op, in, n_in, n_out, LSC_ACT_SILU);
    case LSC_OP_GELU: return compile_activation(op, in, n_in, n_out, LSC_ACT_GELU);
    case LSC_OP_LAYERNORM: return compile_layernorm(op, in, n_in, out, n_out);
    case LSC_OP_SOFTMAX: return compile_softmax(op, in, n_in, n_out);
    case LSC_OP_ADD: return compile_add(op, in, n_in, n_out);
    case LSC_OP_QUANTIZE: {
      if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Quantize needs 1 input and 1 output");
      if (in[0].dtype != LSC_DTYPE_F32)
        return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Quantize: input must be f32");
      op->kind = OpKind::kQuantize;
      op->qdtype = out[0].dtype;
      if (dtype_size(op->qdtype) == 0 || op->qdtype == LSC_DTYPE_F32 || op->qdtype == LSC_DTYPE_F16 ||
          op->qdtype == LSC_DTYPE_F64 || op->qdtype == LSC_DTYPE_I16 || op->qdtype == LSC_DTYPE_I64)
        return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Quantize: output dtype %d", op->qdtype);
      op->kp = 0;
      if (in[0].ndim == 4 && in[0].layout != LSC_LAYOUT_NHWC && out[0].layout == LSC_LAYOUT_NHWC) {
        // relayout to NHWC int8; the output's declared shape gives the stored channel count
        if (!is_int8(op->qdtype) || out[0].ndim != 4 || out[0].quant.count > 1)
          return set_error(LSC_ERROR_UNSUPPORTED_LAYOUT, "Quantize to NHWC: per-tensor int8 output [N,H,W,C] only");
        op->kp = out[0].shape[3];
        if (op->kp % 16 != 0)
          return set_error(LSC_ERROR_INVALID_ARGUMENT, "Quantize to NHWC: stored channels must be a multiple of 16");
        // stride_h = stride_w = b > 1: space-to-depth by b after zero-padding (pad_h, pad_w
        // before; pad + pad_end_delta after)
        op->sh = op->desc.stride_h > 1 ? op->desc.stride_h : 1;
        op->ph = op->sh > 1 ? op->desc.pad_h : 0;
        op->pw = op->sh > 1 ? op->desc.pad_w : 0;
        op->ph_end = op->sh > 1 ? op->desc.pad_h + op->desc.pad_h_end_delta : 0;
        op->pw_end = op->sh > 1 ? op->desc.pad_w + op->desc.pad_w_end_delta : 0;
        if (op->sh > 1 && op->desc.stride_w != op->sh)
          return set_error(LSC_ERROR_INVALID_ARGUMENT, "Quantize space-to-depth needs equal strides");
      }
      return take_qparams(op, out[0]);
    }
    case LSC_OP_DEQUANTIZE: {
      if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Dequantize needs 1 input and 1 output");
      op->kind = OpKind::kDequantize;
      op->qdtype = in[0].dtype;
      if (!(is_int8(op->qdtype) || op->qdtype == LSC_DTYPE_QUINT8 || op->qdtype == LSC_DTYPE_U8 ||
            op->qdtype == LSC_DTYPE_QINT32 || op->qdtype == LSC_DTYPE_I32))
        return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Dequantize: input dtype %d", op->qdtype);
      return take_qparams(op, in[0]);
    }
    default:
      break;
  }
  return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "operator %d (fusion %d, input dtype %d) is not supported by the CUDA backend",
                   op->desc.op_type, op->desc.fusion, n_in > 0 ? in[0].dtype : -1);
}

lsc_status execute_op(lsc_backend* be, const lsc_op* op, const lsc_tensor* in, int n_in,
                      lsc_tensor* out, int n_out, Staging& s) {
  (void)be;
  switch (op->kind) {
    case OpKind::kQGemm: return execute_qgemm(op, in, n_in, out, n_out, s);
    case OpKind::kQuantize: return execute_quant(op, in, n_in, out, n_out, s, true);
    case OpKind::kDequantize: return execute_quant(op, in, n_in, out, n_out, s, false);
    case OpKind::kConvF32:
    case OpKind::kConvI8: return execute_conv(op, in, n_in, out, n_out, s);
    case OpKind::kMatMulF32: return execute_matmul_f32(op, in, n_in, out, n_out, s);
    case OpKind::kFcF32: return execute_fc_f32(op, in, n_in, out, n_out, s);
    case OpKind::kBatchNormF32: return execute_batchnorm(op, in, n_in, out, n_out, s);
    case OpKind::kActF32: return execute_activation(op, in, n_in, out, n_out, s);
    case OpKind::kLayerNorm:
    case OpKind::kSoftmax: return execute_rownorm(op, in, n_in, out, n_out, s);
    case OpKind::kMaxPoolI8:
    case OpKind::kAvgPoolI8:
    case OpKind::kMaxPoolF32:
    case OpKind::kAvgPoolF32: return execute_pool(op, in, n_in, out, n_out, s);
    case OpKind::kAddF32: return execute_add(op, in, n_in, out, n_out, s);
    default: break;
  }
  return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "compiled operator kind %d not executable", static_cast<int>(op->kind));
}

}  // namespace lsc
