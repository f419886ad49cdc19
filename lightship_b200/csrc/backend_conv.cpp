// backend_conv.cpp -- Backend operators for Conv2d (FP32 NCHW and INT8 NHWC), MatMul and
// FullyConnected in FP32, BatchNorm and the standalone activations.
//
// Compile-time weight work (host, f32 rounding of every operation as in the reference):
//   BN fold     f = gamma / sqrt(var + eps); w' = f * w; b' = f * (b - mean) + beta
//               (lightship-core/src/ir/optimizer.rs:727-731)
//   re-layout   OIHW -> [Cout, KH, KW, C] with C padded (K ordered kh, kw, c, like the
//               im2col columns of core/operator/convolution.rs:180-207)
//   FP32        split into TF32 hi + lo parts (contraction_tf32.cu)
//   INT8        per-output-channel symmetric quantization (find_scale_zp + quantize_value,
//               quantization/helpers.rs:101-155); bias_i32 = quantize_value(b', s_a * s_w, 0, QInt32)
#include <math.h>
#include <string.h>

#include <vector>

#include "backend_ops.h"

namespace lsc {
namespace {

const char* tname(const lsc_tensor& t) { return t.name ? t.name : "?"; }

int32_t sat_i32(float v) {
  if (v != v) return 0;
  if (v >= 2147483648.0f) return INT32_MAX;
  if (v <= -2147483648.0f) return INT32_MIN;
  return static_cast<int32_t>(v);
}

void split_host(float x, float& hi, float& lo) {
  uint32_t b;
  memcpy(&b, &x, 4);
  b &= 0xFFFFE000u;
  memcpy(&hi, &b, 4);
  lo = x - hi;
}

int fusion_act(const lsc_op_desc& d) {
  switch (d.fusion) {
    case LSC_FUSION_CONV_RELU:
    case LSC_FUSION_BATCHNORM_RELU:
    case LSC_FUSION_ADD_RELU:
    case LSC_FUSION_MUL_RELU: return LSC_ACT_RELU;
    case LSC_FUSION_CONV_RELU6: return LSC_ACT_RELU6;
    default: return d.activation;
  }
}

float bn_eps(const lsc_op_desc& d) { return d.bn_epsilon > 0.0f ? d.bn_epsilon : 1e-5f; }

lsc_status own_upload(lsc_op* op, const void* host, int64_t bytes, void** dptr) {
  lsc_status st = upload(op->be, host, bytes, dptr);
  if (st == LSC_SUCCESS) op->owned.push_back(*dptr);
  return st;
}

lsc_status read_f32(const lsc_tensor& t, int64_t count, std::vector<float>& out) {
  if (t.dtype != LSC_DTYPE_F32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "tensor '%s' must be f32", tname(t));
  if (numel(t) != count)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "tensor '%s' must hold %lld values", tname(t), (long long)count);
  std::vector<uint8_t> raw;
  lsc_status st = read_tensor_bytes(t, count * 4, raw);
  if (st) return st;
  out.resize(static_cast<size_t>(count));
  if (count) memcpy(out.data(), raw.data(), static_cast<size_t>(count) * 4);
  return LSC_SUCCESS;
}

// Reads conv weights (OIHW f32), optional bias and, for Conv+BatchNorm, folds the BN.
lsc_status conv_weights_f32(lsc_op* op, const lsc_tensor* in, int n_in, std::vector<float>& w,
                            std::vector<float>& b, bool& has_bias) {
  const lsc_tensor& wt = in[1];
  if (wt.ndim != 4) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Conv2d filter '%s' must be 4D OIHW", tname(wt));
  const int64_t co = wt.shape[0], per = wt.shape[1] * wt.shape[2] * wt.shape[3];
  lsc_status st = read_f32(wt, co * per, w);
  if (st) return st;
  has_bias = n_in >= 3 && in[2].data && numel(in[2]) > 0;
  b.assign(static_cast<size_t>(co), 0.0f);
  if (has_bias && (st = read_f32(in[2], co, b))) return st;
  if (op->desc.fusion == LSC_FUSION_CONV_BATCHNORM) {
    if (n_in < 7)
      return set_error(LSC_ERROR_INVALID_ARGUMENT,
                       "Conv+BatchNorm needs inputs X, W, B (may be empty), gamma, beta, mean, var");
    std::vector<float> g, be, mu, var;
    if ((st = read_f32(in[3], co, g)) || (st = read_f32(in[4], co, be)) ||
        (st = read_f32(in[5], co, mu)) || (st = read_f32(in[6], co, var)))
      return st;
    const float eps = bn_eps(op->desc);
    for (int64_t o = 0; o < co; ++o) {
      const float f = g[o] / sqrtf(var[o] + eps);
      for (int64_t i = 0; i < per; ++i) w[o * per + i] = f * w[o * per + i];
      b[o] = f * (b[o] - mu[o]) + be[o];
    }
    has_bias = true;
  }
  return LSC_SUCCESS;
}

// A grouped filter [co, ci_g, kh, kw] (Conv2d::forward with groups, convolution.rs:105-122:
// output channel o belongs to group o / (co / groups) and reads input channels
// [group * ci_g, (group + 1) * ci_g)) as the dense [co, groups * ci_g, kh, kw] filter that is
// zero outside each output channel's group.  The dense convolution then computes the grouped
// one: the zero taps add exact zeros, and the per-output-channel maxima that the weight
// quantization and BN fold read are unchanged.  Costs groups x the MACs of a grouped kernel.
std::vector<float> expand_groups(const std::vector<float>& w, int64_t co, int64_t ci_g, int64_t taps,
                                 int64_t groups) {
  const int64_t ci = ci_g * groups, per_g = ci_g * taps, opg = co / groups;
  std::vector<float> out(static_cast<size_t>(co * ci * taps), 0.0f);
  for (int64_t o = 0; o < co; ++o)
    memcpy(&out[static_cast<size_t>(o * ci * taps + (o / opg) * per_g)], &w[static_cast<size_t>(o * per_g)],
           static_cast<size_t>(per_g) * sizeof(float));
  return out;
}

// OIHW [co, ci, kh, kw] -> [co, kh, kw, cp] (zero channels ci..cp-1).
template <typename T>
std::vector<T> oihw_to_ohwi(const T* w, int64_t co, int64_t ci, int64_t kh, int64_t kw, int64_t cp) {
  std::vector<T> out(static_cast<size_t>(co * kh * kw * cp), T(0));
  for (int64_t o = 0; o < co; ++o)
    for (int64_t c = 0; c < ci; ++c)
      for (int64_t r = 0; r < kh; ++r)
        for (int64_t s = 0; s < kw; ++s)
          out[((o * kh + r) * kw + s) * cp + c] = w[((o * ci + c) * kh + r) * kw + s];
  return out;
}

lsc_status geometry_from(const lsc_op* op, const lsc_tensor& x, bool nhwc, ConvGeometry& g) {
  if (x.ndim != 4) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Conv2d input must be 4D tensor");
  g.n = x.shape[0];
  g.h = nhwc ? x.shape[1] : x.shape[2];
  g.w = nhwc ? x.shape[2] : x.shape[3];
  g.c = op->kp;  // stored channels
  g.c_out = op->n;
  g.kh = op->kh;
  g.kw = op->kw;
  g.sh = op->sh;
  g.sw = op->sw;
  g.ph = op->ph;
  g.pw = op->pw;
  g.dh = op->dh;
  g.dw = op->dw;
  g.ph_b = op->ph_end;
  g.pw_r = op->pw_end;
  const int64_t nh = g.h + g.ph + g.ph_b - g.dh * (g.kh - 1) - 1;
  const int64_t nw = g.w + g.pw + g.pw_r - g.dw * (g.kw - 1) - 1;
  if (nh < 0 || nw < 0) return set_error(LSC_ERROR_SHAPE_MISMATCH, "Conv2d: input smaller than the filter");
  g.oh = nh / g.sh + 1;
  g.ow = nw / g.sw + 1;
  return LSC_SUCCESS;
}

// Pixel grouping of a stride-1 INT8 convolution.  Output group x' (pixels G*x'..G*x'+G-1)
// reads input columns G*x' - pw .. G*x' + G - 2 - pw + KW, i.e. input groups
// x' - ceil(pw/G) .. x' + floor((G + KW - 2 - pw) / G): a kw_g-tap convolution over the
// grouped view with left padding pw_g = ceil(pw/G).
struct PixelGroup {
  int g = 1, kw_g = 0, pw_g = 0;
};

PixelGroup pixel_group_for(int64_t g, int64_t kw, int64_t pw) {
  PixelGroup r;
  r.g = static_cast<int>(g);
  r.pw_g = static_cast<int>((pw + g - 1) / g);
  r.kw_g = static_cast<int>((g + kw - 2 - pw) / g + r.pw_g + 1);
  return r;
}

// Largest G in {8, 4, 2} whose grouped pixel fits one 128-byte im2col request, that at most
// doubles the MMA work (kw_g * G <= 2 * KW; the grouped filter is zero outside each output
// pixel's own taps) and that divides the input and output widths.  1 = no grouping.
int choose_pixel_group(const ConvGeometry& g) {
  if (g.sw != 1 || g.dw != 1 || g.kw < 2) return 1;
  for (int cand : {8, 4, 2}) {
    if (cand * g.c > 128 || g.w % cand || g.ow % cand) continue;
    const PixelGroup pg = pixel_group_for(cand, g.kw, g.pw);
    if (pg.kw_g * cand <= 2 * g.kw) return cand;
  }
  return 1;
}

// The grouped view of geometry g for group G (false when the widths do not divide).
bool grouped_geometry(const lsc_op* op, const ConvGeometry& g, ConvGeometry& gg) {
  const int G = op->group_px;
  if (G <= 1 || g.sw != 1 || g.dw != 1 || g.w % G || g.ow % G) return false;
  gg = g;
  gg.w = g.w / G;
  gg.c = g.c * G;
  gg.c_out = g.c_out * G;
  gg.kw = op->kw_g;
  gg.pw = op->pw_g;
  gg.ow = g.ow / G;
  gg.pw_r = gg.ow - gg.w - gg.pw + gg.kw - 1;
  return true;
}

}  // namespace

// ------------------------------------------------------------------------------ Conv2d
lsc_status compile_conv(lsc_op* op, const lsc_tensor* in, int n_in, const lsc_tensor* out, int n_out) {
  if (n_in < 2 || n_out < 1)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "Conv2d requires 2 inputs (input, filter) and 1 output");
  const lsc_op_desc& d = op->desc;
  if (d.groups < 0) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Conv2d: groups must be positive (got %d)", d.groups);
  if (d.fusion != LSC_FUSION_NONE && d.fusion != LSC_FUSION_CONV_RELU && d.fusion != LSC_FUSION_CONV_RELU6 &&
      d.fusion != LSC_FUSION_CONV_BATCHNORM)
    return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "Conv2d fusion %d is not supported", d.fusion);
  const lsc_tensor& x = in[0];
  const lsc_tensor& wt = in[1];
  if (wt.ndim != 4) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Conv2d filter must be 4D");
  op->sh = d.stride_h > 0 ? d.stride_h : 1;
  op->sw = d.stride_w > 0 ? d.stride_w : 1;
  op->ph = d.pad_h;
  op->pw = d.pad_w;
  op->ph_end = d.pad_h + d.pad_h_end_delta;
  op->pw_end = d.pad_w + d.pad_w_end_delta;
  op->dh = d.dilation_h > 0 ? d.dilation_h : 1;
  op->dw = d.dilation_w > 0 ? d.dilation_w : 1;
  op->act = fusion_act(d);
  const int64_t groups = d.groups > 1 ? d.groups : 1;
  const int64_t co = wt.shape[0];
  if (co % groups != 0)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "Conv2d: %lld output channels do not split into %lld groups",
                     (long long)co, (long long)groups);
  const int64_t ci = wt.shape[1] * groups;  // the filter holds Cin/groups channels per output channel
  op->n = co;
  op->c_in = ci;
  op->kh = wt.shape[2];
  op->kw = wt.shape[3];
  std::vector<float> w, b;
  bool has_bias = false;
  const bool int8 = is_int8(x.dtype);
  if (!int8 && x.dtype != LSC_DTYPE_F32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Conv2d requires F32 or INT8 inputs");
  if (wt.dtype == LSC_DTYPE_F32) {
    lsc_status st = conv_weights_f32(op, in, n_in, w, b, has_bias);
    if (st) return st;
  } else {
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Conv2d filter '%s' must be f32 (quantized at compile for INT8)", tname(wt));
  }
  if (groups > 1) w = expand_groups(w, co, wt.shape[1], op->kh * op->kw, groups);
  const int64_t taps = op->kh * op->kw;
  void* p = nullptr;
  lsc_status st;
  if (!int8) {
    // FP32: NCHW activations; stored channels padded to a multiple of 4
    if (d.pad_h_end_delta != 0 || d.pad_w_end_delta != 0)
      return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "FP32 Conv2d takes symmetric padding only");
    if (x.ndim == 4 && x.shape[1] != ci)
      return set_error(LSC_ERROR_SHAPE_MISMATCH, "Conv2d: input has %lld channels, filter expects %lld",
                       (long long)x.shape[1], (long long)ci);
    op->kind = OpKind::kConvF32;
    op->kp = (ci + 3) / 4 * 4;
    op->winograd = op->fp32_mode == LSC_FP32_WINOGRAD && op->kh == 3 && op->kw == 3 && op->sh == 1 &&
                   op->sw == 1 && op->dh == 1 && op->dw == 1;
    if (op->winograd) {
      // U_xi[o][c] = (G g G^T)[i][j], xi = 4 i + j, G = [1 0 0; 1/2 1/2 1/2; 1/2 -1/2 1/2; 0 0 1]
      // (evaluated in double, rounded once to f32), then split into TF32 halves
      static const double G[4][3] = {{1, 0, 0}, {0.5, 0.5, 0.5}, {0.5, -0.5, 0.5}, {0, 0, 1}};
      const size_t plane = static_cast<size_t>(co * op->kp);
      std::vector<float> hi(16 * plane, 0.0f), lo(16 * plane, 0.0f);
      for (int64_t o = 0; o < co; ++o)
        for (int64_t c = 0; c < ci; ++c) {
          const float* g = &w[static_cast<size_t>((o * ci + c) * 9)];
          double gg[4][3];  // G g
          for (int i = 0; i < 4; ++i)
            for (int j = 0; j < 3; ++j) gg[i][j] = G[i][0] * g[j] + G[i][1] * g[3 + j] + G[i][2] * g[6 + j];
          for (int i = 0; i < 4; ++i)
            for (int j = 0; j < 4; ++j) {
              const float u = static_cast<float>(gg[i][0] * G[j][0] + gg[i][1] * G[j][1] + gg[i][2] * G[j][2]);
              const size_t at = static_cast<size_t>(4 * i + j) * plane + static_cast<size_t>(o * op->kp + c);
              split_host(u, hi[at], lo[at]);
            }
        }
      if ((st = own_upload(op, hi.data(), static_cast<int64_t>(hi.size()) * 4, &op->w))) return st;
      if ((st = own_upload(op, lo.data(), static_cast<int64_t>(lo.size()) * 4, &op->w_lo))) return st;
      if (has_bias) {
        if ((st = own_upload(op, b.data(), co * 4, &p))) return st;
        op->bias_f32 = static_cast<float*>(p);
      }
      return LSC_SUCCESS;
    }
    std::vector<float> wl = oihw_to_ohwi(w.data(), co, ci, op->kh, op->kw, op->kp);
    std::vector<float> hi(wl.size()), lo(wl.size());
    for (size_t i = 0; i < wl.size(); ++i) split_host(wl[i], hi[i], lo[i]);
    const int64_t bytes = static_cast<int64_t>(wl.size()) * 4;
    if ((st = own_upload(op, op->fp32_mode == LSC_FP32_TF32 ? wl.data() : hi.data(), bytes, &op->w))) return st;
    if (op->fp32_mode != LSC_FP32_TF32 && (st = own_upload(op, lo.data(), bytes, &op->w_lo))) return st;
    if (has_bias) {
      if ((st = own_upload(op, b.data(), co * 4, &p))) return st;
      op->bias_f32 = static_cast<float*>(p);
    }
    (void)taps;
    return LSC_SUCCESS;
  }
  // INT8: NHWC activations with C stored as a multiple of 16
  if (x.ndim != 4) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Conv2d input must be 4D NHWC");
  const int64_t cs = x.shape[3];
  if (cs % 16 != 0 || cs < ci)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "INT8 Conv2d: NHWC input must store >= %lld channels, a multiple of 16 (got %lld)",
                     (long long)ci, (long long)cs);
  op->kind = OpKind::kConvI8;
  op->kp = cs;
  const float s_a = x.quant.count > 0 && x.quant.scale ? x.quant.scale[0] : 1.0f;
  // per output channel: [kh, kw, ci] values, symmetric int8
  std::vector<float> wk = oihw_to_ohwi(w.data(), co, ci, op->kh, op->kw, ci);
  const int64_t per = taps * ci;
  std::vector<int8_t> q(static_cast<size_t>(co * per));
  std::vector<float> sw(static_cast<size_t>(co)), scale(static_cast<size_t>(co));
  for (int64_t o = 0; o < co; ++o) {
    float mn = INFINITY, mx = -INFINITY;
    for (int64_t i = 0; i < per; ++i) {
      mn = fminf(mn, wk[o * per + i]);
      mx = fmaxf(mx, wk[o * per + i]);
    }
    const float am = fmaxf(fabsf(mx), fabsf(mn));
    const float s = am > 0.0f ? am / 127.0f : 1.0f;
    sw[o] = s;
    for (int64_t i = 0; i < per; ++i) {
      int32_t v = sat_i32(roundf(wk[o * per + i] / s));
      q[o * per + i] = static_cast<int8_t>(v < -128 ? -128 : (v > 127 ? 127 : v));
    }
    scale[o] = s_a * s;
  }
  // [co, kh, kw, ci] -> [co, kh, kw, cs]
  std::vector<int8_t> qp(static_cast<size_t>(co * taps * cs), 0);
  for (int64_t o = 0; o < co; ++o)
    for (int64_t t = 0; t < taps; ++t) memcpy(&qp[(o * taps + t) * cs], &q[(o * taps + t) * ci], static_cast<size_t>(ci));
  if ((st = own_upload(op, qp.data(), co * taps * cs, &op->w))) return st;
  if ((st = own_upload(op, scale.data(), co * 4, &p))) return st;
  op->scale = static_cast<float*>(p);
  std::vector<int32_t> bi;
  if (has_bias) {
    bi.resize(static_cast<size_t>(co));
    for (int64_t o = 0; o < co; ++o) bi[o] = sat_i32(roundf(b[o] / scale[o]));
    if ((st = own_upload(op, bi.data(), co * 4, &p))) return st;
    op->bias_i32 = static_cast<int32_t*>(p);
  }
  // pixel-grouped filter for the compile-time input width
  ConvGeometry g0{};
  if ((st = geometry_from(op, x, true, g0))) return st;
  const int G = choose_pixel_group(g0);
  if (G > 1) {
    const PixelGroup pg = pixel_group_for(G, op->kw, op->pw);
    op->group_px = G;
    op->kw_g = pg.kw_g;
    op->pw_g = pg.pw_g;
    const int64_t kg = op->kh * pg.kw_g * G * cs;  // grouped K per output column
    std::vector<int8_t> wg(static_cast<size_t>(G * co * kg), 0);
    for (int gi = 0; gi < G; ++gi)
      for (int64_t o = 0; o < co; ++o)
        for (int64_t ky = 0; ky < op->kh; ++ky)
          for (int kx_g = 0; kx_g < pg.kw_g; ++kx_g)
            for (int sp = 0; sp < G; ++sp) {
              const int64_t kx = static_cast<int64_t>(G) * (kx_g - pg.pw_g) + sp - gi + op->pw;
              if (kx < 0 || kx >= op->kw) continue;
              memcpy(&wg[static_cast<size_t>((gi * co + o) * kg + ((ky * pg.kw_g + kx_g) * G + sp) * cs)],
                     &qp[static_cast<size_t>(((o * op->kh + ky) * op->kw + kx) * cs)], static_cast<size_t>(cs));
            }
    if ((st = own_upload(op, wg.data(), static_cast<int64_t>(wg.size()), &op->w_grouped))) return st;
    std::vector<float> sg(static_cast<size_t>(G * co));
    for (int gi = 0; gi < G; ++gi) memcpy(&sg[gi * co], scale.data(), static_cast<size_t>(co) * 4);
    if ((st = own_upload(op, sg.data(), G * co * 4, &p))) return st;
    op->scale_grouped = static_cast<float*>(p);
    if (has_bias) {
      std::vector<int32_t> bg(static_cast<size_t>(G * co));
      for (int gi = 0; gi < G; ++gi) memcpy(&bg[gi * co], bi.data(), static_cast<size_t>(co) * 4);
      if ((st = own_upload(op, bg.data(), G * co * 4, &p))) return st;
      op->bias_grouped = static_cast<int32_t*>(p);
    }
  }
  op->s_out = 1.0f;
  for (int i = 0; i < n_out; ++i) {
    if (is_int8(out[i].dtype)) {
      float so = d.output_scale;
      if (!(so > 0.0f) && out[i].quant.count > 0 && out[i].quant.scale) so = out[i].quant.scale[0];
      if (!(so > 0.0f))
        return set_error(LSC_ERROR_INVALID_ARGUMENT, "int8 output '%s' needs an output scale", tname(out[i]));
      op->s_out = so;
    } else if (out[i].dtype != LSC_DTYPE_F32 && out[i].dtype != LSC_DTYPE_I32 && out[i].dtype != LSC_DTYPE_QINT32) {
      return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "output '%s': dtype %d", tname(out[i]), out[i].dtype);
    }
  }
  return LSC_SUCCESS;
}

lsc_status execute_conv(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                        int n_out, Staging& s) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Conv2d: missing tensors");
  const lsc_tensor& x = in[0];
  const bool int8 = op->kind == OpKind::kConvI8;
  ConvGeometry g{};
  lsc_status st = geometry_from(op, x, int8, g);
  if (st) return st;
  if (!int8) {
    if (x.dtype != LSC_DTYPE_F32) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Conv2d requires F32 inputs");
    if (x.shape[1] != op->c_in)
      return set_error(LSC_ERROR_SHAPE_MISMATCH, "Conv2d: input has %lld channels, filter expects %lld",
                       (long long)x.shape[1], (long long)op->c_in);
    const int64_t hw = g.h * g.w;
    const void* xd = nullptr;
    if ((st = s.input(x, g.n * op->c_in * hw * 4, &xd))) return st;
    if (op->winograd) {
      lsc_tensor& y = out[0];
      if (y.dtype != LSC_DTYPE_F32) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Conv2d output must be F32");
      void* yd = nullptr;
      if ((st = s.output(y, g.n * g.c_out * g.oh * g.ow * 4, &yd))) return st;
      set_shape(y, {g.n, g.c_out, g.oh, g.ow});
      ConvGeometry gw = g;
      gw.c = op->c_in;
      float* scratch = static_cast<float*>(s.scratch(winograd_f32_scratch_floats(gw, op->kp, true) * 4));
      if (!scratch) return LSC_ERROR_OUT_OF_MEMORY;
      return launch_conv_winograd_f32(static_cast<const float*>(xd), static_cast<const float*>(op->w),
                                      static_cast<const float*>(op->w_lo), gw, op->kp, op->bias_f32, op->act,
                                      static_cast<float*>(yd), scratch, true, s.st);
    }
    const bool split = op->fp32_mode != LSC_FP32_TF32;
    const int64_t nbytes = g.n * hw * g.c * 4;
    float* hi = static_cast<float*>(s.scratch(nbytes));
    float* lo = split ? static_cast<float*>(s.scratch(nbytes)) : nullptr;
    if (!hi || (split && !lo)) return LSC_ERROR_OUT_OF_MEMORY;
    if ((st = prep_split_nchw_to_nhwc(static_cast<const float*>(xd), g.n, op->c_in, hw, g.c, hi, lo, s.st))) return st;
    lsc_tensor& y = out[0];
    if (y.dtype != LSC_DTYPE_F32) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Conv2d output must be F32");
    void* yd = nullptr;
    if ((st = s.output(y, g.n * g.c_out * g.oh * g.ow * 4, &yd))) return st;
    set_shape(y, {g.n, g.c_out, g.oh, g.ow});
    const int64_t ks_floats = tf32_conv_ksplit_floats(g);
    float* ks_ws = ks_floats > 0 ? static_cast<float*>(s.scratch(ks_floats * 4)) : nullptr;
    return launch_conv_tf32(hi, lo, static_cast<const float*>(op->w), static_cast<const float*>(op->w_lo), g,
                            op->bias_f32, op->act, static_cast<float*>(yd), split, s.st, ks_ws,
                            ks_ws ? ks_floats : 0);
  }
  if (!is_int8(x.dtype)) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "INT8 Conv2d: input must be int8 NHWC");
  if (x.shape[3] != op->kp)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "INT8 Conv2d: input stores %lld channels, compiled for %lld",
                     (long long)x.shape[3], (long long)op->kp);
  const void* xd = nullptr;
  if ((st = s.input(x, g.n * g.h * g.w * g.c, &xd))) return st;
  int8_t* o_i8 = nullptr;
  float* o_f32 = nullptr;
  int32_t* o_i32 = nullptr;
  float s_out = op->s_out;
  const int64_t m = g.n * g.oh * g.ow;
  for (int i = 0; i < n_out; ++i) {
    void* dptr = nullptr;
    if ((st = s.output(out[i], m * g.c_out * dtype_size(out[i].dtype), &dptr))) return st;
    if (is_int8(out[i].dtype)) {
      o_i8 = static_cast<int8_t*>(dptr);
      // a calibrated output scale carried by the output tensor overrides the compiled one
      if (out[i].quant.count > 0 && out[i].quant.scale && out[i].quant.scale[0] > 0.0f)
        s_out = out[i].quant.scale[0];
    } else if (out[i].dtype == LSC_DTYPE_F32) {
      o_f32 = static_cast<float*>(dptr);
    } else {
      o_i32 = static_cast<int32_t*>(dptr);
    }
    set_shape(out[i], {g.n, g.oh, g.ow, g.c_out});
  }
  // optional residual (execute-time input 1): int8 NHWC shaped like the output, added before
  // the activation -- a BasicBlock's Add+ReLU fused into its second convolution
  const void* rd = nullptr;
  float r_scale = 1.0f;
  if (n_in >= 2 && in[1].data) {
    const lsc_tensor& r = in[1];
    if (!is_int8(r.dtype)) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Conv2d residual must be int8");
    if (numel(r) != m * g.c_out)
      return set_error(LSC_ERROR_SHAPE_MISMATCH, "Conv2d residual '%s' must match the output shape", tname(r));
    if ((st = s.input(r, m * g.c_out, &rd))) return st;
    r_scale = r.quant.count > 0 && r.quant.scale ? r.quant.scale[0] : 1.0f;
  }
  ConvGeometry gg{};
  if (grouped_geometry(op, g, gg))
    return launch_conv_i8(static_cast<const int8_t*>(xd), static_cast<const int8_t*>(op->w_grouped), gg,
                          op->bias_grouped, op->scale_grouped, s_out, op->act, op->rounding, o_i8, o_f32, o_i32,
                          static_cast<const int8_t*>(rd), r_scale, s.st);
  return launch_conv_i8(static_cast<const int8_t*>(xd), static_cast<const int8_t*>(op->w), g, op->bias_i32,
                        op->scale, s_out, op->act, op->rounding, o_i8, o_f32, o_i32,
                        static_cast<const int8_t*>(rd), r_scale, s.st);
}

lsc_status execute_conv_pool(const lsc_op* op, const lsc_tensor& x, lsc_tensor& y, cudaStream_t st) {
  if (op->kind != OpKind::kConvI8 || op->act != LSC_ACT_RELU || !op->w_grouped)
    return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "conv + max pool: a pixel-grouped INT8 ReLU convolution only");
  if (!is_int8(x.dtype) || x.ndim != 4 || x.shape[3] != op->kp || x.location != LSC_MEM_DEVICE ||
      y.location != LSC_MEM_DEVICE || !is_int8(y.dtype))
    return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "conv + max pool: device int8 NHWC tensors only");
  ConvGeometry g{};
  lsc_status s = geometry_from(op, x, true, g);
  if (s) return s;
  ConvGeometry gg{};
  if (!grouped_geometry(op, g, gg))
    return set_error(LSC_ERROR_UNSUPPORTED_OPERATOR, "conv + max pool: the convolution does not run pixel-grouped here");
  const int64_t bytes = g.n * (g.oh / 2) * (g.ow / 2) * g.c_out;
  if (y.nbytes && y.nbytes < static_cast<uint64_t>(bytes))
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "conv + max pool: output '%s' needs %lld bytes", tname(y), (long long)bytes);
  const float s_out = y.quant.count > 0 && y.quant.scale && y.quant.scale[0] > 0.0f ? y.quant.scale[0] : op->s_out;
  s = launch_conv_pool_i8(static_cast<const int8_t*>(x.data), static_cast<const int8_t*>(op->w_grouped), gg,
                          op->group_px, op->bias_grouped, op->scale_grouped, s_out, op->act, op->rounding,
                          static_cast<int8_t*>(y.data), st);
  if (s == LSC_SUCCESS) set_shape(y, {g.n, g.oh / 2, g.ow / 2, g.c_out});
  return s;
}

// ------------------------------------------------------------------------------ pooling (INT8 NHWC)
lsc_status compile_pool(lsc_op* op, const lsc_tensor* in, int n_in, int n_out, bool global) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Missing input or output");
  const bool f32 = in[0].dtype == LSC_DTYPE_F32;
  if (!is_int8(in[0].dtype) && !f32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "pooling on the CUDA backend takes int8 NHWC or f32 NCHW input");
  const lsc_op_desc& d = op->desc;
  if (f32)
    op->kind = global ? OpKind::kAvgPoolF32 : OpKind::kMaxPoolF32;
  else
    op->kind = global ? OpKind::kAvgPoolI8 : OpKind::kMaxPoolI8;
  op->kh = d.kernel_h > 0 ? d.kernel_h : 1;
  op->kw = d.kernel_w > 0 ? d.kernel_w : 1;
  if (!global && (d.pad_h < 0 || d.pad_w < 0 || d.pad_h >= op->kh || d.pad_w >= op->kw))
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "MaxPool2d: padding must be smaller than the window");
  op->sh = d.stride_h > 0 ? d.stride_h : 1;
  op->sw = d.stride_w > 0 ? d.stride_w : 1;
  op->ph = d.pad_h;
  op->pw = d.pad_w;
  op->s_out = d.output_scale;
  return LSC_SUCCESS;
}

lsc_status execute_pool(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                        int n_out, Staging& s) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Missing input or output");
  const lsc_tensor& x = in[0];
  if (op->kind == OpKind::kMaxPoolF32 || op->kind == OpKind::kAvgPoolF32) {
    // f32 NCHW (Pool2d, operator/pooling.rs): [N, C, OH, OW] max, [N, C, 1, 1] global average
    if (x.dtype != LSC_DTYPE_F32 || x.ndim != 4)
      return set_error(LSC_ERROR_INVALID_ARGUMENT, "pooling takes a 4D f32 NCHW input here");
    const int64_t n = x.shape[0], c = x.shape[1], h = x.shape[2], w = x.shape[3];
    const void* xd = nullptr;
    void* yd = nullptr;
    lsc_status st = s.input(x, n * c * h * w * 4, &xd);
    if (st) return st;
    if (out[0].dtype != LSC_DTYPE_F32) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "pooling output must be f32");
    if (op->kind == OpKind::kAvgPoolF32) {
      if ((st = s.output(out[0], n * c * 4, &yd))) return st;
      set_shape(out[0], {n, c, 1, 1});
      return launch_avgpool_f32(static_cast<const float*>(xd), static_cast<float*>(yd), n, c, h * w, s.st);
    }
    const int64_t oh = (h + 2 * op->ph - op->kh) / op->sh + 1, ow = (w + 2 * op->pw - op->kw) / op->sw + 1;
    if (oh <= 0 || ow <= 0) return set_error(LSC_ERROR_SHAPE_MISMATCH, "MaxPool2d: window larger than the input");
    if ((st = s.output(out[0], n * c * oh * ow * 4, &yd))) return st;
    set_shape(out[0], {n, c, oh, ow});
    return launch_maxpool_f32(static_cast<const float*>(xd), static_cast<float*>(yd), n, c, h, w, oh, ow,
                              static_cast<int>(op->kh), static_cast<int>(op->kw), op->sh, op->sw, op->ph, op->pw,
                              s.st);
  }
  if (!is_int8(x.dtype) || x.ndim != 4)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "pooling takes a 4D int8 NHWC input");
  const int64_t n = x.shape[0], h = x.shape[1], w = x.shape[2], c = x.shape[3];
  const void* xd = nullptr;
  lsc_status st = s.input(x, n * h * w * c, &xd);
  if (st) return st;
  if (op->kind == OpKind::kMaxPoolI8) {
    const int64_t oh = (h + 2 * op->ph - op->kh) / op->sh + 1, ow = (w + 2 * op->pw - op->kw) / op->sw + 1;
    if (oh <= 0 || ow <= 0) return set_error(LSC_ERROR_SHAPE_MISMATCH, "MaxPool2d: window larger than the input");
    void* yd = nullptr;
    if ((st = s.output(out[0], n * oh * ow * c, &yd))) return st;
    set_shape(out[0], {n, oh, ow, c});
    return launch_maxpool_i8(static_cast<const int8_t*>(xd), static_cast<int8_t*>(yd), n, h, w, c, oh, ow,
                             static_cast<int>(op->kh), static_cast<int>(op->kw), op->sh, op->sw, op->ph, op->pw, s.st);
  }
  const float s_in = x.quant.count > 0 && x.quant.scale ? x.quant.scale[0] : 1.0f;
  int8_t* o_i8 = nullptr;
  float* o_f32 = nullptr;
  float s_out = op->s_out;
  for (int i = 0; i < n_out; ++i) {
    void* yd = nullptr;
    if ((st = s.output(out[i], n * c * dtype_size(out[i].dtype), &yd))) return st;
    set_shape(out[i], {n, c});
    if (out[i].dtype == LSC_DTYPE_F32) {
      o_f32 = static_cast<float*>(yd);
    } else if (is_int8(out[i].dtype)) {
      o_i8 = static_cast<int8_t*>(yd);
      if (out[i].quant.count > 0 && out[i].quant.scale && out[i].quant.scale[0] > 0.0f)
        s_out = out[i].quant.scale[0];
      if (!(s_out > 0.0f))
        return set_error(LSC_ERROR_INVALID_ARGUMENT, "GlobalAvgPool2d: int8 output needs an output scale");
    } else {
      return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "GlobalAvgPool2d output must be f32 or int8");
    }
  }
  return launch_avgpool_i8(static_cast<const int8_t*>(xd), n, h * w, c, s_in, s_out, op->rounding, o_i8, o_f32, s.st);
}

// ------------------------------------------------------------------------------ MatMul / FC
lsc_status compile_matmul_f32(lsc_op* op, const lsc_tensor* in, int n_in, int n_out) {
  if (n_in < 2 || n_out < 1)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "MatMul requires 2 inputs and 1 output");
  if (in[0].dtype != LSC_DTYPE_F32 || in[1].dtype != LSC_DTYPE_F32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "MatMul requires F32 inputs");
  op->kind = OpKind::kMatMulF32;
  op->act = op->desc.activation;
  return LSC_SUCCESS;
}

lsc_status execute_matmul_f32(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                              int n_out, Staging& s) {
  if (n_in < 2 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "MatMul requires 2 inputs and 1 output");
  const lsc_tensor& a = in[0];
  const lsc_tensor& b = in[1];
  if (a.dtype != LSC_DTYPE_F32 || b.dtype != LSC_DTYPE_F32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "MatMul requires F32 inputs");
  if (a.ndim != 2 || b.ndim != 2) return set_error(LSC_ERROR_INVALID_ARGUMENT, "MatMul requires 2D matrices");
  const int64_t m = a.shape[0], k = a.shape[1], kb = b.shape[0], n = b.shape[1];
  if (k != kb)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "Matrix dimension mismatch: A_cols=%lld != B_rows=%lld",
                     (long long)k, (long long)kb);
  lsc_tensor& c = out[0];
  if (c.dtype != LSC_DTYPE_F32) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "MatMul output must be F32");
  const void* ad = nullptr;
  const void* bd = nullptr;
  void* cd = nullptr;
  lsc_status st;
  if ((st = s.input(a, m * k * 4, &ad)) || (st = s.input(b, k * n * 4, &bd)) || (st = s.output(c, m * n * 4, &cd)))
    return st;
  set_shape(c, {m, n});
  if (m == 0 || n == 0) return LSC_SUCCESS;
  if (k == 0) {
    LSC_CUDA_TRY(cudaMemsetAsync(cd, 0, static_cast<size_t>(m * n * 4), s.st));
    return LSC_SUCCESS;
  }
  const bool split = op->fp32_mode != LSC_FP32_TF32;
  const int64_t kp = (k + 3) / 4 * 4;
  float* ah = static_cast<float*>(s.scratch(m * kp * 4));
  float* al = split ? static_cast<float*>(s.scratch(m * kp * 4)) : nullptr;
  float* bh = static_cast<float*>(s.scratch(n * kp * 4));
  float* bl = split ? static_cast<float*>(s.scratch(n * kp * 4)) : nullptr;
  if (!ah || !bh || (split && (!al || !bl))) return LSC_ERROR_OUT_OF_MEMORY;
  if ((st = prep_split_rows(static_cast<const float*>(ad), m, k, kp, ah, al, s.st))) return st;
  if ((st = prep_split_transpose(static_cast<const float*>(bd), k, n, kp, bh, bl, s.st))) return st;
  const int64_t ks_floats = tf32_gemm_ksplit_floats(m, n, kp);
  float* ks_ws = ks_floats > 0 ? static_cast<float*>(s.scratch(ks_floats * 4)) : nullptr;
  return launch_gemm_tf32(ah, al, bh, bl, m, n, kp, nullptr, op->act, static_cast<float*>(cd), n, split, s.st, ks_ws,
                          ks_ws ? ks_floats : 0);
}

lsc_status compile_fc_f32(lsc_op* op, const lsc_tensor* in, int n_in, int n_out) {
  if (n_in < 2 || n_out < 1)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "FullyConnected requires 2 inputs (input, weight) and 1 output");
  const lsc_tensor& x = in[0];
  const lsc_tensor& w = in[1];
  if (x.dtype != LSC_DTYPE_F32 || w.dtype != LSC_DTYPE_F32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "FullyConnected requires F32 inputs");
  if (w.ndim != 2 || (x.ndim == 2 && x.shape[1] != w.shape[1]))
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "Weight in_features != input in_features");
  const int64_t n = w.shape[0], k = w.shape[1];
  std::vector<float> wf;
  lsc_status st = read_f32(w, n * k, wf);
  if (st) return st;
  const int64_t kp = (k + 3) / 4 * 4;
  std::vector<float> hi(static_cast<size_t>(n * kp), 0.0f), lo(static_cast<size_t>(n * kp), 0.0f);
  const bool split = op->fp32_mode != LSC_FP32_TF32;
  for (int64_t i = 0; i < n; ++i)
    for (int64_t j = 0; j < k; ++j) {
      if (split) split_host(wf[i * k + j], hi[i * kp + j], lo[i * kp + j]);
      else hi[i * kp + j] = wf[i * k + j];
    }
  if ((st = own_upload(op, hi.data(), n * kp * 4, &op->w))) return st;
  if (split && (st = own_upload(op, lo.data(), n * kp * 4, &op->w_lo))) return st;
  if (n_in >= 3 && in[2].data && numel(in[2]) > 0) {
    std::vector<float> b;
    if ((st = read_f32(in[2], n, b))) return st;
    void* p = nullptr;
    if ((st = own_upload(op, b.data(), n * 4, &p))) return st;
    op->bias_f32 = static_cast<float*>(p);
  }
  op->kind = OpKind::kFcF32;
  op->n = n;
  op->k = k;
  op->kp = kp;
  op->act = op->desc.activation;
  return LSC_SUCCESS;
}

lsc_status execute_fc_f32(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                          int n_out, Staging& s) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "FullyConnected: missing tensors");
  const lsc_tensor& x = in[0];
  if (x.dtype != LSC_DTYPE_F32) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "FullyConnected requires F32 inputs");
  if (x.ndim != 2) return set_error(LSC_ERROR_INVALID_ARGUMENT, "FullyConnected requires 2D input and weight");
  if (x.shape[1] != op->k)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "Weight in_features %lld != input in_features %lld",
                     (long long)op->k, (long long)x.shape[1]);
  const int64_t m = x.shape[0];
  const void* xd = nullptr;
  void* yd = nullptr;
  lsc_status st;
  if ((st = s.input(x, m * op->k * 4, &xd)) || (st = s.output(out[0], m * op->n * 4, &yd))) return st;
  set_shape(out[0], {m, op->n});
  if (m == 0) return LSC_SUCCESS;
  const bool split = op->fp32_mode != LSC_FP32_TF32;
  float* xh = static_cast<float*>(s.scratch(m * op->kp * 4));
  float* xl = split ? static_cast<float*>(s.scratch(m * op->kp * 4)) : nullptr;
  if (!xh || (split && !xl)) return LSC_ERROR_OUT_OF_MEMORY;
  if ((st = prep_split_rows(static_cast<const float*>(xd), m, op->k, op->kp, xh, xl, s.st))) return st;
  const int64_t ks_floats = tf32_gemm_ksplit_floats(m, op->n, op->kp);
  float* ks_ws = ks_floats > 0 ? static_cast<float*>(s.scratch(ks_floats * 4)) : nullptr;
  return launch_gemm_tf32(xh, xl, static_cast<const float*>(op->w), static_cast<const float*>(op->w_lo), m,
                          op->n, op->kp, op->bias_f32, op->act, static_cast<float*>(yd), op->n, split, s.st, ks_ws,
                          ks_ws ? ks_floats : 0);
}

// ------------------------------------------------------------------------------ BatchNorm / activations
lsc_status compile_batchnorm(lsc_op* op, const lsc_tensor* in, int n_in, int n_out) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Missing input or output");
  const lsc_tensor& x = in[0];
  if (x.dtype != LSC_DTYPE_F32) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "BatchNorm requires F32 input");
  if (x.ndim < 2) return set_error(LSC_ERROR_INVALID_ARGUMENT, "BatchNorm requires at least 2D input");
  const int64_t c = x.shape[1];
  // parameters (X, gamma, beta, mean, var) or the reference's defaults (batchnorm.rs:178-187)
  std::vector<float> g(static_cast<size_t>(c), 1.0f), be(static_cast<size_t>(c), 0.0f),
      mu(static_cast<size_t>(c), 0.0f), var(static_cast<size_t>(c), 1.0f);
  lsc_status st;
  if (n_in >= 5) {
    if ((st = read_f32(in[1], c, g)) || (st = read_f32(in[2], c, be)) || (st = read_f32(in[3], c, mu)) ||
        (st = read_f32(in[4], c, var)))
      return st;
  }
  const float eps = bn_eps(op->desc);
  std::vector<float> inv(static_cast<size_t>(c));
  for (int64_t i = 0; i < c; ++i) {
    const float sd = sqrtf(var[i] + eps);
    inv[i] = 1.0f / sd;
  }
  // packed per-channel vectors: gamma | beta | mean | inv_std
  std::vector<float> pk(static_cast<size_t>(4 * c));
  memcpy(&pk[0], g.data(), c * 4);
  memcpy(&pk[c], be.data(), c * 4);
  memcpy(&pk[2 * c], mu.data(), c * 4);
  memcpy(&pk[3 * c], inv.data(), c * 4);
  void* p = nullptr;
  if ((st = own_upload(op, pk.data(), 4 * c * 4, &p))) return st;
  op->bias_f32 = static_cast<float*>(p);
  op->n = c;
  op->kind = OpKind::kBatchNormF32;
  op->act = op->desc.fusion == LSC_FUSION_BATCHNORM_RELU ? LSC_ACT_RELU : op->desc.activation;
  return LSC_SUCCESS;
}

lsc_status execute_batchnorm(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                             int n_out, Staging& s) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Missing input or output");
  const lsc_tensor& x = in[0];
  if (x.dtype != LSC_DTYPE_F32) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "BatchNorm requires F32 input");
  if (x.ndim < 2 || x.shape[1] != op->n)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "Channel mismatch: expected %lld", (long long)op->n);
  const int64_t total = numel(x);
  int64_t spatial = 1;
  for (int i = 2; i < x.ndim; ++i) spatial *= x.shape[i];
  const void* xd = nullptr;
  void* yd = nullptr;
  lsc_status st;
  if ((st = s.input(x, total * 4, &xd)) || (st = s.output(out[0], total * 4, &yd))) return st;
  out[0].ndim = x.ndim;
  for (int i = 0; i < x.ndim; ++i) out[0].shape[i] = x.shape[i];
  const float* pk = op->bias_f32;
  const int64_t c = op->n;
  return launch_batchnorm_f32(static_cast<const float*>(xd), static_cast<float*>(yd), x.shape[0], c, spatial,
                              pk, pk + c, pk + 2 * c, pk + 3 * c, op->act, s.st);
}

lsc_status compile_activation(lsc_op* op, const lsc_tensor* in, int n_in, int n_out, int act) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Missing input or output");
  if (in[0].dtype != LSC_DTYPE_F32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "activation requires F32 input");
  op->kind = OpKind::kActF32;
  op->act = act;
  return LSC_SUCCESS;
}

// Add (OperatorType::Add, backend/cpu.rs:468-517): y = a + b elementwise on equal shapes,
// then the activation (FusionType::AddReLU, or the descriptor's activation).
lsc_status compile_add(lsc_op* op, const lsc_tensor* in, int n_in, int n_out) {
  if (n_in < 2 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Add requires 2 inputs and 1 output");
  if (in[0].dtype != LSC_DTYPE_F32 || in[1].dtype != LSC_DTYPE_F32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Add requires F32 inputs");
  op->kind = OpKind::kAddF32;
  op->act = op->desc.fusion == LSC_FUSION_ADD_RELU ? LSC_ACT_RELU : op->desc.activation;
  if (op->act < LSC_ACT_NONE || op->act > LSC_ACT_GELU)
    return set_error(LSC_ERROR_INVALID_ARGUMENT, "Add: bad activation %d", op->act);
  return LSC_SUCCESS;
}

lsc_status execute_add(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out, int n_out, Staging& s) {
  if (n_in < 2 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Add requires 2 inputs and 1 output");
  const lsc_tensor& a = in[0];
  const lsc_tensor& b = in[1];
  if (a.dtype != LSC_DTYPE_F32 || b.dtype != LSC_DTYPE_F32 || out[0].dtype != LSC_DTYPE_F32)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Add requires F32 tensors");
  const int64_t total = numel(a);
  if (total < 0 || numel(b) != total)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "Add: inputs hold %lld and %lld elements", (long long)total,
                     (long long)numel(b));
  const void* ad = nullptr;
  const void* bd = nullptr;
  void* yd = nullptr;
  lsc_status st;
  if ((st = s.input(a, total * 4, &ad)) || (st = s.input(b, total * 4, &bd)) ||
      (st = s.output(out[0], total * 4, &yd)))
    return st;
  out[0].ndim = a.ndim;
  for (int i = 0; i < a.ndim; ++i) out[0].shape[i] = a.shape[i];
  return launch_add_f32(static_cast<const float*>(ad), static_cast<const float*>(bd), static_cast<float*>(yd), total,
                        op->act, s.st);
}

lsc_status execute_activation(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out,
                              int n_out, Staging& s) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Missing input or output");
  const lsc_tensor& x = in[0];
  if (x.dtype != LSC_DTYPE_F32) return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "activation requires F32 input");
  const int64_t total = numel(x);
  if (total < 0) return set_error(LSC_ERROR_SHAPE_MISMATCH, "bad shape");
  const void* xd = nullptr;
  void* yd = nullptr;
  lsc_status st;
  if ((st = s.input(x, total * 4, &xd)) || (st = s.output(out[0], total * 4, &yd))) return st;
  out[0].ndim = x.ndim;
  for (int i = 0; i < x.ndim; ++i) out[0].shape[i] = x.shape[i];
  return launch_activation_f32(static_cast<const float*>(xd), static_cast<float*>(yd), total, op->act, s.st);
}

// ------------------------------------------------------------------------------ LayerNorm / Softmax
// LayerNorm (operator/layernorm.rs:59-205): inputs (x, gamma?, beta?) with gamma / beta of the
// last axis's length, epsilon from bn_epsilon (0 -> the reference's 1e-5).  Softmax
// (operator/softmax.rs:37-169): the last axis (SoftmaxAxis::Last, the reference's default).
// Both keep the input's storage type (f32 or f16) and shape.
// An int8 output (QInt8, one scale, zero point 0) makes the kernel quantize the normalised
// row as a following Quantize operator would (helpers.rs:138-156); its scale is fixed here.
lsc_status compile_layernorm(lsc_op* op, const lsc_tensor* in, int n_in, const lsc_tensor* out, int n_out) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "LayerNorm: missing input or output");
  const lsc_tensor& x = in[0];
  if (x.dtype != LSC_DTYPE_F32 && x.dtype != LSC_DTYPE_F16)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "LayerNorm requires F32 or F16 input");
  if (x.ndim < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "LayerNorm requires at least 1D input");
  op->kind = OpKind::kLayerNorm;
  op->qdtype = x.dtype;
  op->q_channels = 0;
  if (is_int8(out[0].dtype)) {
    const lsc_quant& q = out[0].quant;
    if (q.count != 1 || !q.scale || !(q.scale[0] > 0.0f))
      return set_error(LSC_ERROR_INVALID_ARGUMENT, "LayerNorm: int8 output '%s' needs one scale > 0", tname(out[0]));
    if (q.zero_point && q.zero_point[0] != 0)
      return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "LayerNorm: int8 output must be symmetric (zero point 0)");
    op->q_channels = 1;  // marks the quantized output
    op->q_scale0 = q.scale[0];
  } else if (out[0].dtype != x.dtype) {
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "LayerNorm: output dtype must match the input or be int8");
  }
  const int64_t d = x.shape[x.ndim - 1];
  op->n = d;
  op->s_out = bn_eps(op->desc);
  lsc_status st;
  void* p = nullptr;
  if (n_in >= 2 && in[1].data) {
    std::vector<float> g;
    if ((st = read_f32(in[1], d, g)) || (st = own_upload(op, g.data(), d * 4, &p))) return st;
    op->scale = static_cast<float*>(p);
  }
  if (n_in >= 3 && in[2].data) {
    std::vector<float> b;
    if ((st = read_f32(in[2], d, b)) || (st = own_upload(op, b.data(), d * 4, &p))) return st;
    op->bias_f32 = static_cast<float*>(p);
  }
  return LSC_SUCCESS;
}

lsc_status compile_softmax(lsc_op* op, const lsc_tensor* in, int n_in, int n_out) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "Softmax: missing input or output");
  const lsc_tensor& x = in[0];
  if (x.dtype != LSC_DTYPE_F32 && x.dtype != LSC_DTYPE_F16)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "Softmax requires F32 or F16 input");
  op->kind = OpKind::kSoftmax;
  op->qdtype = x.dtype;
  return LSC_SUCCESS;
}

lsc_status execute_rownorm(const lsc_op* op, const lsc_tensor* in, int n_in, lsc_tensor* out, int n_out,
                           Staging& s) {
  if (n_in < 1 || n_out < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "missing input or output");
  const lsc_tensor& x = in[0];
  const bool ln = op->kind == OpKind::kLayerNorm;
  if (x.dtype != op->qdtype)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "%s: input dtype %d, compiled for %d", ln ? "LayerNorm" : "Softmax",
                     x.dtype, op->qdtype);
  if (x.ndim < 1) return set_error(LSC_ERROR_INVALID_ARGUMENT, "input must be at least 1D");
  const int64_t d = x.shape[x.ndim - 1];
  if (ln && d != op->n)
    return set_error(LSC_ERROR_SHAPE_MISMATCH, "LayerNorm: last axis %lld, compiled for %lld", (long long)d,
                     (long long)op->n);
  const int64_t total = numel(x);
  if (total < 0) return set_error(LSC_ERROR_SHAPE_MISMATCH, "bad shape");
  const int64_t esz = dtype_size(x.dtype);
  const bool quantized = ln && op->q_channels == 1;
  if (quantized ? !is_int8(out[0].dtype) : out[0].dtype != x.dtype)
    return set_error(LSC_ERROR_UNSUPPORTED_DATATYPE, "output dtype %d does not match the compiled operator",
                     out[0].dtype);
  const void* xd = nullptr;
  void* yd = nullptr;
  lsc_status st;
  if ((st = s.input(x, total * esz, &xd)) || (st = s.output(out[0], total * (quantized ? 1 : esz), &yd))) return st;
  out[0].ndim = x.ndim;
  for (int i = 0; i < x.ndim; ++i) out[0].shape[i] = x.shape[i];
  const int64_t rows = d > 0 ? total / d : 0;
  if (quantized)
    return launch_layernorm(xd, nullptr, x.dtype, rows, d, op->scale, op->bias_f32, op->s_out, s.st,
                            static_cast<int8_t*>(yd), op->q_scale0, op->rounding);
  if (ln) return launch_layernorm(xd, yd, x.dtype, rows, d, op->scale, op->bias_f32, op->s_out, s.st);
  return launch_softmax(xd, yd, x.dtype, rows, d, s.st);
}

}  // namespace lsc
