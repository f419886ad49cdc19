// lsc_oracle.cpp -- CPU restatement of LightShip's dense-contraction math.
//
// TEST INFRASTRUCTURE ONLY (see lsc_oracle.h).  Built with -ffp-contract=off.
// Citations are reference-project paths: core/ = lightship-core/src/.
#include "lsc_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

extern "C" const char* orc_version(void) { return "lsc-oracle 1"; }

namespace {

// Rust `f32 as i32`: saturating, NaN -> 0.
inline int32_t rust_f32_to_i32(float v) {
  if (v != v) return 0;
  if (v >= 2147483648.0f) return INT32_MAX;
  if (v <= -2147483648.0f) return INT32_MIN;
  return (int32_t)v;
}

// Rust `f32::clamp(lo, hi)`: NaN passes through; -0.0 is not < 0.0.
inline float rust_clamp(float x, float lo, float hi) {
  float r = x;
  if (r < lo) r = lo;
  if (r > hi) r = hi;
  return r;
}

// Rust `f32 as i8` after a clamp to [-128,127]: NaN -> 0, otherwise truncation.
inline int8_t rust_f32_to_i8(float v) {
  if (v != v) return 0;
  if (v >= 127.0f) return 127;
  if (v <= -128.0f) return -128;
  return (int8_t)(int)v;
}

void conv_i8_chain_impl(const int8_t* x, const int8_t* w, int64_t n, int64_t h, int64_t wd,
                        int64_t c_in, int64_t c_out, int64_t kh, int64_t kw, int64_t sh,
                        int64_t sw, int64_t ph, int64_t pw, int64_t dh, int64_t dw,
                        int64_t groups, const int32_t* bias, const float* scale, int act,
                        float s_out, int rounding, const int8_t* residual, float r_scale,
                        int8_t* out_i8, float* out_f32, int32_t* out_acc, int threads);

inline int threads_or_default(int t) {
#ifdef _OPENMP
  return t > 0 ? t : omp_get_max_threads();
#else
  (void)t;
  return 1;
#endif
}

}  // namespace

extern "C" {

// ---------------------------------------------------------------------------
// FP32 GEMM
// ---------------------------------------------------------------------------

// core/platform/simd.rs:588-598 (gemm_scalar): per element a sequential f32 sum over k,
// each product rounded before the add, then added into C.
void orc_gemm_scalar(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      float sum = 0.0f;
      for (int64_t p = 0; p < k; ++p) sum += a[i * k + p] * b[p * n + j];
      c[i * n + j] += sum;
    }
}

// core/platform/simd.rs:1938-2052 (gemm_neon) and :2055-2085 (gemm_neon_simple).
// For m*n < 512 the simple path is a sequential k sum (the lane-0 products of its vector
// code are exactly a[k]*b[k][j] added in k order).  Otherwise K is cut in kc=128 blocks and,
// per block, each C element receives a fresh sequential partial sum over that block.
void orc_gemm_blocked(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k) {
  if (m * n < 512) {
    orc_gemm_scalar(a, b, c, m, n, k);
    return;
  }
  const int64_t mc = std::min<int64_t>(64, m);
  const int64_t kc = std::min<int64_t>(128, k);
  if (kc == 0) return;
  for (int64_t kb = 0; kb < k; kb += kc) {
    const int64_t ke = std::min(kb + kc, k);
    for (int64_t mb = 0; mb < m; mb += mc) {
      const int64_t me = std::min(mb + mc, m);
      for (int64_t i = mb; i < me; ++i) {
        int64_t j = 0;
        for (; j + 16 <= n; j += 16) {
          float s[16];
          for (int t = 0; t < 16; ++t) s[t] = 0.0f;
          for (int64_t p = kb; p < ke; ++p) {
            const float av = a[i * k + p];
            const float* bp = b + p * n + j;
            for (int t = 0; t < 16; ++t) s[t] += av * bp[t];
          }
          for (int t = 0; t < 16; ++t) c[i * n + j + t] += s[t];
        }
        for (; j < n; ++j) {
          float s = 0.0f;
          for (int64_t p = kb; p < ke; ++p) s += a[i * k + p] * b[p * n + j];
          c[i * n + j] += s;
        }
      }
    }
  }
}

// core/backend/cpu.rs:949-1063 with core/cpu/thread_scheduler.rs:352-386: C is zeroed, the
// M*N output is cut into contiguous element ranges of max(M*N/threads, N) elements, each
// range widened to whole rows and computed with the blocked kernel.  Per-element values do
// not depend on the split (every row is computed whole), so rows are simply partitioned.
void orc_matmul(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                int threads) {
  memset(c, 0, sizeof(float) * (size_t)(m * n));
  const int nt = threads_or_default(threads);
  if (nt <= 1 || m * n <= 1024) {
    orc_gemm_blocked(a, b, c, m, n, k);
    return;
  }
  const int64_t total = m * n;
  const int64_t block = std::max<int64_t>(total / nt, n);
  std::vector<std::pair<int64_t, int64_t>> rows;
  for (int64_t s = 0; s < total; s += block) {
    const int64_t e = std::min(s + block, total);
    int64_t r0 = s / n, r1 = (e + n - 1) / n;
    if (!rows.empty()) r0 = std::max(r0, rows.back().second);
    if (r1 > r0) rows.push_back({r0, r1});
  }
#pragma omp parallel for num_threads(nt) schedule(static, 1)
  for (int64_t t = 0; t < (int64_t)rows.size(); ++t) {
    const int64_t r0 = rows[t].first, r1 = rows[t].second;
    orc_gemm_blocked(a + r0 * k, b, c + r0 * n, r1 - r0, n, k);
  }
}

// core/backend/cpu.rs:1209-1290: sequential f32 sum over in_features, no bias.
void orc_fully_connected(const float* x, const float* w, float* y, int64_t batch, int64_t in_f,
                         int64_t out_f, int threads) {
  const int nt = threads_or_default(threads);
#pragma omp parallel for num_threads(nt) collapse(2) schedule(static)
  for (int64_t bi = 0; bi < batch; ++bi)
    for (int64_t o = 0; o < out_f; ++o) {
      float sum = 0.0f;
      for (int64_t i = 0; i < in_f; ++i) sum += x[bi * in_f + i] * w[o * in_f + i];
      y[bi * out_f + o] = sum;
    }
}

// ---------------------------------------------------------------------------
// Conv2d
// ---------------------------------------------------------------------------

// core/operator/convolution.rs:55-62, computed in signed arithmetic.
int64_t orc_conv_out_dim(int64_t in, int64_t k, int64_t stride, int64_t pad, int64_t dil) {
  const int64_t num = in + 2 * pad - dil * (k - 1) - 1;
  if (num < 0 || stride <= 0) return -1;
  return num / stride + 1;
}

namespace {
// One image of Conv2d::forward (convolution.rs:161-240): im2col with ki ordered (kh,kw,c),
// explicit transpose, gemm_simd(filter[c_out_pg,K], col_t[K,P]) and NCHW scatter.
// `korder_ref` selects the reference's filter flattening (c,kh,kw) (convolution.rs:245-267);
// the default pairs the filter in the same (kh,kw,c) order as the columns.
void conv_one_image(const float* x, const float* w, float* y, int64_t c_in, int64_t h,
                    int64_t wd, int64_t c_out, int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                    int64_t ph, int64_t pw, int64_t dh, int64_t dw, int64_t groups,
                    int64_t oh, int64_t ow, bool korder_ref) {
  const int64_t cpg = c_in / groups, opg = c_out / groups;
  const int64_t K = kh * kw * cpg, P = oh * ow;
  std::vector<float> col((size_t)(K * P)), col_t((size_t)(K * P)), filt((size_t)(opg * K)),
      out((size_t)(opg * P));
  for (int64_t g = 0; g < groups; ++g) {
    for (int64_t o = 0; o < opg; ++o) {
      const int64_t go = g * opg + o;
      int64_t ki = 0;
      if (korder_ref) {
        for (int64_t c = 0; c < cpg; ++c)
          for (int64_t r = 0; r < kh; ++r)
            for (int64_t s = 0; s < kw; ++s) filt[o * K + ki++] = w[((go * cpg + c) * kh + r) * kw + s];
      } else {
        for (int64_t r = 0; r < kh; ++r)
          for (int64_t s = 0; s < kw; ++s)
            for (int64_t c = 0; c < cpg; ++c) filt[o * K + ki++] = w[((go * cpg + c) * kh + r) * kw + s];
      }
    }
    for (int64_t yy = 0; yy < oh; ++yy)
      for (int64_t xx = 0; xx < ow; ++xx) {
        const int64_t base = (yy * ow + xx) * K;
        int64_t ki = 0;
        for (int64_t r = 0; r < kh; ++r)
          for (int64_t s = 0; s < kw; ++s)
            for (int64_t c = 0; c < cpg; ++c) {
              const int64_t iy = yy * sh + r * dh - ph, ix = xx * sw + s * dw - pw;
              const bool ok = iy >= 0 && iy < h && ix >= 0 && ix < wd;
              col[base + ki++] = ok ? x[((g * cpg + c) * h + iy) * wd + ix] : 0.0f;
            }
      }
    for (int64_t i = 0; i < K; ++i)
      for (int64_t j = 0; j < P; ++j) col_t[i * P + j] = col[j * K + i];
    std::fill(out.begin(), out.end(), 0.0f);
    orc_gemm_blocked(filt.data(), col_t.data(), out.data(), opg, P, K);
    for (int64_t o = 0; o < opg; ++o)
      memcpy(y + (g * opg + o) * P, out.data() + o * P, sizeof(float) * (size_t)P);
  }
}
}  // namespace

void orc_conv2d_nchw(const float* x, const float* w, const float* bias, float* y, int64_t n,
                     int64_t c_in, int64_t h, int64_t wd, int64_t c_out, int64_t kh, int64_t kw,
                     int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh, int64_t dw,
                     int64_t groups, int threads) {
  const int64_t oh = orc_conv_out_dim(h, kh, sh, ph, dh), ow = orc_conv_out_dim(wd, kw, sw, pw, dw);
  if (oh <= 0 || ow <= 0) return;
  const int nt = threads_or_default(threads);
#pragma omp parallel for num_threads(nt) schedule(static, 1)
  for (int64_t b = 0; b < n; ++b) {
    conv_one_image(x + b * c_in * h * wd, w, y + b * c_out * oh * ow, c_in, h, wd, c_out, kh, kw,
                   sh, sw, ph, pw, dh, dw, groups, oh, ow, false);
    if (bias)
      for (int64_t o = 0; o < c_out; ++o)
        for (int64_t p = 0; p < oh * ow; ++p) y[(b * c_out + o) * oh * ow + p] += bias[o];
  }
}

void orc_conv2d_nchw_reference_korder(const float* x, const float* w, float* y, int64_t n,
                                      int64_t c_in, int64_t h, int64_t wd, int64_t c_out,
                                      int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                                      int64_t pw, int64_t dh, int64_t dw, int64_t groups) {
  const int64_t oh = orc_conv_out_dim(h, kh, sh, ph, dh), ow = orc_conv_out_dim(wd, kw, sw, pw, dw);
  if (oh <= 0 || ow <= 0) return;
  for (int64_t b = 0; b < n; ++b)
    conv_one_image(x + b * c_in * h * wd, w, y + b * c_out * oh * ow, c_in, h, wd, c_out, kh, kw,
                   sh, sw, ph, pw, dh, dw, groups, oh, ow, true);
}

// ---------------------------------------------------------------------------
// BatchNorm, BN fold, activations
// ---------------------------------------------------------------------------

// core/operator/batchnorm.rs:154-215: std = sqrt(var+eps); inv = 1/std;
// y = gamma*((x-mean)*inv) + beta, per channel.  Indexing uses the NCHW channel of each
// element (the reference's c*n*spatial start is only right for N=1).
void orc_batchnorm_inference(const float* x, float* y, int64_t n, int64_t c, int64_t spatial,
                             const float* gamma, const float* beta, const float* mean,
                             const float* var, float eps) {
  for (int64_t ci = 0; ci < c; ++ci) {
    const float g = gamma ? gamma[ci] : 1.0f, be = beta ? beta[ci] : 0.0f;
    const float mu = mean ? mean[ci] : 0.0f, v = var ? var[ci] : 1.0f;
    const float sd = sqrtf(v + eps);
    const float inv = 1.0f / sd;
    for (int64_t b = 0; b < n; ++b) {
      const float* xs = x + (b * c + ci) * spatial;
      float* ys = y + (b * c + ci) * spatial;
      for (int64_t i = 0; i < spatial; ++i) {
        const float xn = (xs[i] - mu) * inv;
        ys[i] = g * xn + be;
      }
    }
  }
}

// core/ir/optimizer.rs:727-731.  f = gamma / sqrt(var + eps); w' = f*w; b' = f*(b-mean)+beta.
void orc_bn_fold(const float* w, const float* bias, const float* gamma, const float* beta,
                 const float* mean, const float* var, float eps, int64_t c_out, int64_t per_out,
                 float* w_out, float* b_out) {
  for (int64_t o = 0; o < c_out; ++o) {
    const float f = gamma[o] / sqrtf(var[o] + eps);
    for (int64_t i = 0; i < per_out; ++i) w_out[o * per_out + i] = f * w[o * per_out + i];
    const float b = bias ? bias[o] : 0.0f;
    b_out[o] = f * (b - mean[o]) + beta[o];
  }
}

// ReLU: core/platform/simd.rs:552-556 (x > 0 ? x : 0, so NaN and -0 give +0).
// ReLU6: simd.rs:558-562 (f32::clamp(0, 6): NaN and -0 pass through).
// SiLU: core/operator/silu.rs:47-61 (x > 20 -> x; x < -20 -> 0; else x / (1 + exp(-x))),
// exp being the platform libm expf that Rust's f32::exp lowers to.
float orc_act(float x, int act) {
  switch (act) {
    case ORC_ACT_RELU: return x > 0.0f ? x : 0.0f;
    case ORC_ACT_RELU6: return rust_clamp(x, 0.0f, 6.0f);
    case ORC_ACT_SILU:
      if (x > 20.0f) return x;
      if (x < -20.0f) return 0.0f;
      return x / (1.0f + expf(-x));
    case ORC_ACT_GELU: {
      // Gelu::tanh_gelu with its polynomial tanh_approx (core/operator/gelu.rs:77-103)
      const float sqrt_2_over_pi = 0.7978845608f;
      const float c = 0.044715f;
      const float x_cube = x * x * x;
      const float t = sqrt_2_over_pi * (x + c * x_cube);
      float th;
      if (t > 5.0f) {
        th = 1.0f;
      } else if (t < -5.0f) {
        th = -1.0f;
      } else {
        const float t2 = t * t, t3 = t2 * t, t5 = t3 * t2, t7 = t5 * t2;
        th = t - t3 / 3.0f + t5 / 5.0f - t7 / 7.0f;
      }
      return 0.5f * x * (1.0f + th);
    }
    default: return x;
  }
}

void orc_act_inplace(float* x, int64_t n, int act) {
  for (int64_t i = 0; i < n; ++i) x[i] = orc_act(x[i], act);
}

// LayerNorm::normalize_simd (core/operator/layernorm.rs:153-205) per row: mean = sum / d,
// variance = sum((x - mean)^2) / d, std = sqrt(variance + eps), y = (x - mean) / std, then
// gamma * y and + beta.  Sums run in index order in f32 (the reference's horizontal_sum
// order differs by lane; the comparison is against a stated tolerance).
void orc_layernorm(const float* x, float* y, int64_t rows, int64_t d, const float* gamma,
                   const float* beta, float eps) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * d;
    float* yr = y + r * d;
    if (d == 0) continue;
    float s = 0.0f;
    for (int64_t i = 0; i < d; ++i) s += xr[i];
    const float mean = s / static_cast<float>(d);
    float sq = 0.0f;
    for (int64_t i = 0; i < d; ++i) {
      const float t = xr[i] - mean;
      sq += t * t;
    }
    const float var = sq / static_cast<float>(d);
    const float sd = sqrtf(var + eps);
    for (int64_t i = 0; i < d; ++i) {
      float v = (xr[i] - mean) / sd;
      if (gamma) v = gamma[i] * v;
      if (beta) v += beta[i];
      yr[i] = v;
    }
  }
}

// Softmax::compute (core/operator/softmax.rs:106-146) per row: max by f32::max, sum of
// exp(x - max) in index order, y = exp(x - max) * (1 / sum); a row whose sum is not positive
// is left as it is.
void orc_softmax(const float* x, float* y, int64_t rows, int64_t d) {
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * d;
    float* yr = y + r * d;
    for (int64_t i = 0; i < d; ++i) yr[i] = xr[i];
    if (d == 0) continue;
    float mx = -INFINITY;
    for (int64_t i = 0; i < d; ++i) mx = fmaxf(mx, xr[i]);
    float s = 0.0f;
    for (int64_t i = 0; i < d; ++i) s += expf(xr[i] - mx);
    if (s > 0.0f) {
      const float scale = 1.0f / s;
      for (int64_t i = 0; i < d; ++i) yr[i] = expf(xr[i] - mx) * scale;
    }
  }
}

// ---------------------------------------------------------------------------
// Quantization
// ---------------------------------------------------------------------------

// half-away = Rust f32::round (helpers.rs:153, quantized_ops.rs:45) = C roundf;
// half-even = rintf under the default round-to-nearest-even mode.
float orc_round(float x, int rounding) {
  return rounding == ORC_ROUND_HALF_EVEN ? rintf(x) : roundf(x);
}

static void qrange(int qdtype, int32_t* lo, int32_t* hi) {
  switch (qdtype) {
    case ORC_QINT8: *lo = -128; *hi = 127; break;
    case ORC_QINT32: *lo = INT32_MIN; *hi = INT32_MAX; break;
    default: *lo = 0; *hi = 255; break;  // QUInt8 and the reference's `_` arm
  }
}

// helpers.rs:139-155: ((value/scale).round() as i32 + zero_point).clamp(qmin, qmax); the
// i32 add wraps as in a Rust release build.
int32_t orc_quantize_value(float value, float scale, int32_t zero_point, int qdtype) {
  int32_t lo, hi;
  qrange(qdtype, &lo, &hi);
  const int32_t r = rust_f32_to_i32(roundf(value / scale));
  const int32_t q = (int32_t)((uint32_t)r + (uint32_t)zero_point);
  return q < lo ? lo : (q > hi ? hi : q);
}

// helpers.rs:158-160: (q as f32 - zp as f32) * scale.
float orc_dequantize_value(int32_t q, float scale, int32_t zero_point) {
  return ((float)q - (float)zero_point) * scale;
}

// helpers.rs:101-136.  min/max fold with f32::min/max (NaN ignored), then
// symmetric: s = absmax/qmax (1.0 if absmax == 0), zp = 0;
// asymmetric: s = (max-min)/(qmax-qmin) (1.0 if max <= min), zp = round(qmin - min/s).
int orc_find_scale_zp(const float* data, int64_t n, int qdtype, int symmetric, float* scale,
                      int32_t* zero_point) {
  if (n <= 0) {
    *scale = 1.0f;  // QuantizationParameters::default() (scheme.rs:123-127)
    *zero_point = 0;
    return 0;
  }
  float mn = INFINITY, mx = -INFINITY;
  for (int64_t i = 0; i < n; ++i) {
    mn = fminf(mn, data[i]);
    mx = fmaxf(mx, data[i]);
  }
  int32_t qmin, qmax;
  qrange(qdtype, &qmin, &qmax);
  if (symmetric) {
    const float am = fmaxf(fabsf(mx), fabsf(mn));
    *scale = am > 0.0f ? am / (float)qmax : 1.0f;
    *zero_point = 0;
  } else {
    // (qmax - qmin) is an i32 subtraction in the reference; it wraps for QInt32.
    const int32_t span = (int32_t)((uint32_t)qmax - (uint32_t)qmin);
    const float s = mx > mn ? (mx - mn) / (float)span : 1.0f;
    const float z = (float)qmin - mn / s;
    *scale = s;
    *zero_point = rust_f32_to_i32(roundf(z));
  }
  return 1;
}

// helpers.rs:11-50 (per-tensor; QInt8 bytes are `v as i8 as u8`, QUInt8 `v as u8`).
void orc_quantize_tensor(const float* x, int64_t n, float scale, int32_t zp, int qdtype,
                         void* out) {
  for (int64_t i = 0; i < n; ++i) {
    const int32_t q = orc_quantize_value(x[i], scale, zp, qdtype);
    if (qdtype == ORC_QINT8) ((int8_t*)out)[i] = (int8_t)q;
    else if (qdtype == ORC_QINT32) ((int32_t*)out)[i] = q;
    else ((uint8_t*)out)[i] = (uint8_t)q;
  }
}

// helpers.rs:53-94.
void orc_dequantize_tensor(const void* q, int64_t n, float scale, int32_t zp, int qdtype,
                           float* out) {
  for (int64_t i = 0; i < n; ++i) {
    int32_t v;
    if (qdtype == ORC_QINT8) v = ((const int8_t*)q)[i];
    else if (qdtype == ORC_QINT32) v = ((const int32_t*)q)[i];
    else v = ((const uint8_t*)q)[i];
    out[i] = orc_dequantize_value(v, scale, zp);
  }
}

// quantized_ops.rs:43-48: (x/s).round().clamp(-128,127) as i8, with R selectable.
void orc_quantize_sym(const float* x, int8_t* q, int64_t n, float scale, int rounding) {
  for (int64_t i = 0; i < n; ++i)
    q[i] = rust_f32_to_i8(rust_clamp(orc_round(x[i] / scale, rounding), -128.0f, 127.0f));
}

void orc_quantize_weights_per_channel(const float* w, int64_t rows, int64_t cols, int8_t* q,
                                      float* scales) {
  for (int64_t r = 0; r < rows; ++r) {
    float s;
    int32_t zp;
    orc_find_scale_zp(w + r * cols, cols, ORC_QINT8, 1, &s, &zp);
    scales[r] = s;
    for (int64_t c = 0; c < cols; ++c)
      q[r * cols + c] = (int8_t)orc_quantize_value(w[r * cols + c], s, 0, ORC_QINT8);
  }
}

// ---------------------------------------------------------------------------
// INT8 chain
// ---------------------------------------------------------------------------

// quantized_ops.rs:13-33 (NN layout, i32 accumulate; the scales are unused there).
void orc_gemm_i8_nn(const int8_t* a, const int8_t* b, int32_t* c, int64_t m, int64_t n,
                    int64_t k, int threads) {
  const int nt = threads_or_default(threads);
#pragma omp parallel for num_threads(nt) schedule(static)
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      int32_t s = 0;
      for (int64_t p = 0; p < k; ++p) s += (int32_t)a[i * k + p] * (int32_t)b[p * n + j];
      c[i * n + j] = s;
    }
}

void orc_gemm_i8_tn(const int8_t* a, const int8_t* w, int32_t* c, int64_t m, int64_t n,
                    int64_t k, int threads) {
  const int nt = threads_or_default(threads);
#pragma omp parallel for num_threads(nt) schedule(static)
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      const int8_t* ar = a + i * k;
      const int8_t* wr = w + j * k;
      int32_t s = 0;
      for (int64_t p = 0; p < k; ++p) s += (int32_t)ar[p] * (int32_t)wr[p];
      c[i * n + j] = s;
    }
}

namespace {
inline void epilogue_one(int32_t acc, int32_t bias, float scale, int act, float s_out,
                         int rounding, int8_t* oi8, float* of32, int32_t* oacc,
                         const int8_t* res = nullptr, float r_scale = 1.0f) {
  acc = (int32_t)((uint32_t)acc + (uint32_t)bias);  // i32 add (wrapping)
  float y = (float)acc * scale;                      // dequantize, quantized_ops.rs:36-40
  if (res) y = y + orc_dequantize_value(*res, r_scale, 0);  // residual, dequantized
  y = orc_act(y, act);
  if (of32) *of32 = y;
  if (oacc) *oacc = acc;
  if (oi8) *oi8 = rust_f32_to_i8(rust_clamp(orc_round(y / s_out, rounding), -128.0f, 127.0f));
}
}  // namespace

void orc_requant(const int32_t* acc, int64_t m, int64_t n, const int32_t* bias,
                 const float* scale, int act, float s_out, int rounding, int8_t* out_i8,
                 float* out_f32, int32_t* out_acc) {
  for (int64_t i = 0; i < m; ++i)
    for (int64_t j = 0; j < n; ++j) {
      const int64_t e = i * n + j;
      epilogue_one(acc[e], bias ? bias[j] : 0, scale[j], act, s_out, rounding,
                   out_i8 ? out_i8 + e : nullptr, out_f32 ? out_f32 + e : nullptr,
                   out_acc ? out_acc + e : nullptr);
    }
}

void orc_gemm_i8_chain(const int8_t* a, const int8_t* w, int64_t m, int64_t n, int64_t k,
                       const int32_t* bias, const float* scale, int act, float s_out,
                       int rounding, int8_t* out_i8, float* out_f32, int32_t* out_acc,
                       int threads) {
  const int nt = threads_or_default(threads);
#pragma omp parallel for num_threads(nt) schedule(static)
  for (int64_t i = 0; i < m; ++i) {
    const int8_t* ar = a + i * k;
    for (int64_t j = 0; j < n; ++j) {
      const int8_t* wr = w + j * k;
      int32_t s = 0;
      for (int64_t p = 0; p < k; ++p) s += (int32_t)ar[p] * (int32_t)wr[p];
      const int64_t e = i * n + j;
      epilogue_one(s, bias ? bias[j] : 0, scale[j], act, s_out, rounding,
                   out_i8 ? out_i8 + e : nullptr, out_f32 ? out_f32 + e : nullptr,
                   out_acc ? out_acc + e : nullptr);
    }
  }
}

void orc_conv2d_i8_nhwc_chain(const int8_t* x, const int8_t* w, int64_t n, int64_t h,
                              int64_t wd, int64_t c_in, int64_t c_out, int64_t kh, int64_t kw,
                              int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh,
                              int64_t dw, int64_t groups, const int32_t* bias,
                              const float* scale, int act, float s_out, int rounding,
                              int8_t* out_i8, float* out_f32, int32_t* out_acc, int threads) {
  conv_i8_chain_impl(x, w, n, h, wd, c_in, c_out, kh, kw, sh, sw, ph, pw, dh, dw, groups, bias,
                     scale, act, s_out, rounding, nullptr, 1.0f, out_i8, out_f32, out_acc, threads);
}

void orc_conv2d_i8_nhwc_chain_res(const int8_t* x, const int8_t* w, int64_t n, int64_t h,
                                  int64_t wd, int64_t c_in, int64_t c_out, int64_t kh, int64_t kw,
                                  int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t dh,
                                  int64_t dw, const int32_t* bias, const float* scale, int act,
                                  float s_out, int rounding, const int8_t* residual,
                                  float r_scale, int8_t* out_i8, float* out_f32, int32_t* out_acc,
                                  int threads) {
  conv_i8_chain_impl(x, w, n, h, wd, c_in, c_out, kh, kw, sh, sw, ph, pw, dh, dw, 1, bias, scale,
                     act, s_out, rounding, residual, r_scale, out_i8, out_f32, out_acc, threads);
}

// quantize_value (helpers.rs:139-155) per element with R selectable, NCHW -> NHWC, zero pad.
void orc_quantize_nchw_to_nhwc(const float* x, int8_t* y, int64_t n, int64_t c, int64_t hw,
                               int64_t cp, float scale, int rounding) {
  for (int64_t b = 0; b < n; ++b)
    for (int64_t p = 0; p < hw; ++p)
      for (int64_t ch = 0; ch < cp; ++ch) {
        int8_t q = 0;
        if (ch < c) {
          const int32_t r = rust_f32_to_i32(orc_round(x[(b * c + ch) * hw + p] / scale, rounding));
          q = (int8_t)(r < -128 ? -128 : (r > 127 ? 127 : r));
        }
        y[(b * hw + p) * cp + ch] = q;
      }
}

void orc_maxpool_i8_nhwc(const int8_t* x, int8_t* y, int64_t n, int64_t h, int64_t w, int64_t c,
                         int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw) {
  const int64_t oh = (h + 2 * ph - kh) / sh + 1, ow = (w + 2 * pw - kw) / sw + 1;
  for (int64_t b = 0; b < n; ++b)
    for (int64_t oy = 0; oy < oh; ++oy)
      for (int64_t ox = 0; ox < ow; ++ox)
        for (int64_t ch = 0; ch < c; ++ch) {
          int m = -128;
          for (int64_t r = 0; r < kh; ++r) {
            const int64_t iy = oy * sh - ph + r;
            if (iy < 0 || iy >= h) continue;
            for (int64_t s = 0; s < kw; ++s) {
              const int64_t ix = ox * sw - pw + s;
              if (ix < 0 || ix >= w) continue;
              const int v = x[((b * h + iy) * w + ix) * c + ch];
              m = v > m ? v : m;
            }
          }
          y[((b * oh + oy) * ow + ox) * c + ch] = (int8_t)m;
        }
}

void orc_avgpool_i8_nhwc(const int8_t* x, int64_t n, int64_t hw, int64_t c, float s_in,
                         float s_out, int rounding, int8_t* y_i8, float* y_f32) {
  for (int64_t b = 0; b < n; ++b)
    for (int64_t ch = 0; ch < c; ++ch) {
      int32_t sum = 0;
      for (int64_t p = 0; p < hw; ++p) sum += x[(b * hw + p) * c + ch];
      const float v = ((float)sum * s_in) / (float)hw;
      if (y_f32) y_f32[b * c + ch] = v;
      if (y_i8) {
        const int32_t r = rust_f32_to_i32(orc_round(v / s_out, rounding));
        y_i8[b * c + ch] = (int8_t)(r < -128 ? -128 : (r > 127 ? 127 : r));
      }
    }
}

}  // extern "C"

namespace {
void conv_i8_chain_impl(const int8_t* x, const int8_t* w, int64_t n, int64_t h, int64_t wd,
                        int64_t c_in, int64_t c_out, int64_t kh, int64_t kw, int64_t sh,
                        int64_t sw, int64_t ph, int64_t pw, int64_t dh, int64_t dw,
                        int64_t groups, const int32_t* bias, const float* scale, int act,
                        float s_out, int rounding, const int8_t* residual, float r_scale,
                        int8_t* out_i8, float* out_f32, int32_t* out_acc, int threads) {
  const int64_t oh = orc_conv_out_dim(h, kh, sh, ph, dh), ow = orc_conv_out_dim(wd, kw, sw, pw, dw);
  if (oh <= 0 || ow <= 0) return;
  const int64_t cpg = c_in / groups, opg = c_out / groups;
  const int nt = threads_or_default(threads);
#pragma omp parallel for num_threads(nt) collapse(2) schedule(static)
  for (int64_t b = 0; b < n; ++b)
    for (int64_t yy = 0; yy < oh; ++yy)
      for (int64_t xx = 0; xx < ow; ++xx)
        for (int64_t o = 0; o < c_out; ++o) {
          const int64_t g = o / opg;
          int32_t s = 0;
          for (int64_t r = 0; r < kh; ++r) {
            const int64_t iy = yy * sh + r * dh - ph;
            if (iy < 0 || iy >= h) continue;
            for (int64_t q = 0; q < kw; ++q) {
              const int64_t ix = xx * sw + q * dw - pw;
              if (ix < 0 || ix >= wd) continue;
              const int8_t* xp = x + ((b * h + iy) * wd + ix) * c_in + g * cpg;
              const int8_t* wp = w + ((o * kh + r) * kw + q) * cpg;
              for (int64_t c = 0; c < cpg; ++c) s += (int32_t)xp[c] * (int32_t)wp[c];
            }
          }
          const int64_t e = ((b * oh + yy) * ow + xx) * c_out + o;
          epilogue_one(s, bias ? bias[o] : 0, scale[o], act, s_out, rounding,
                       out_i8 ? out_i8 + e : nullptr, out_f32 ? out_f32 + e : nullptr,
                       out_acc ? out_acc + e : nullptr, residual ? residual + e : nullptr, r_scale);
        }
}
}  // namespace
