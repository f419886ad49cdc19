// epilogue.cuh -- the INT8 chain's per-element epilogue, written to give the same bits as
// LightShip's CPU math:
//   acc += bias[n]                         (i32, wrapping)
//   y    = (f32)acc * scale[n]             dequantize   core/cpu/quantized_ops.rs:36-40
//   y    = act(y)                          ReLU         core/platform/simd.rs:552-556
//                                          ReLU6        core/platform/simd.rs:558-562
//                                          SiLU         core/operator/silu.rs:47-61
//   q    = (i8)clamp(R(y / s_out), -128, 127)           core/cpu/quantized_ops.rs:43-48
// Every operation is an explicitly rounded intrinsic so nvcc cannot contract it into an
// FMA or replace the IEEE division.
#pragma once
#include <stdint.h>

#include "lightship_cuda.h"

namespace lsc {

__device__ __forceinline__ float act_relu(float x) { return x > 0.0f ? x : 0.0f; }

// Rust f32::clamp(0, 6): NaN (with its payload) and -0.0 pass through unchanged.  The NaN
// test comes first so the compiler cannot lower the clamp to min/max instructions, which
// return the canonical NaN.
__device__ __forceinline__ float act_relu6(float x) {
  if (x != x) return x;
  float r = x;
  if (r < 0.0f) r = 0.0f;
  if (r > 6.0f) r = 6.0f;
  return r;
}

// 2^(i/32) for the libm-equivalent expf below (bits, exponent field lowered by i/32).
static __device__ const uint64_t kExpfTab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

// expf as the host's libm computes it, so that SiLU matches Rust's f32::exp (which lowers to
// the platform expf: glibc on Linux) bit for bit.  The method is the table-driven exp2f design
// of Szabolcs Nagy in ARM's optimized-routines, which glibc (sysdeps/ieee754/flt-32/e_expf.c,
// since 2.28) and musl use: with N = 32, k = round(x * N / ln2) (by adding 1.5 * 2^52),
// r = x * N / ln2 - k in [-1/2, 1/2], exp(x) = 2^(k/N) * 2^(r/N) where 2^(k/N) is the table
// entry 2^((k mod N)/N) with k/N added to its exponent, and 2^(r/N) ~ 1 + c2 r + c1 r^2 + c0 r^3,
// all in double, rounded once to float.  The coefficients are the published polynomial
// (ln2-based, scaled by 1/N^i); the table holds 2^(i/32) correctly rounded to double with
// i * 2^52 / 32 subtracted from its bits.  Valid for |x| < 88 (SiLU needs |x| <= 20).
// Checked on every float in [-20, 20] against glibc's expf (tests/expf_check.c), and on the
// device through the SiLU operator against the oracle.
__device__ __forceinline__ float expf_libm(float x) {
  constexpr double kInvLn2N = 0x1.71547652b82fep+0 * 32;
  constexpr double kShift = 0x1.8p+52;
  constexpr double kC0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;
  constexpr double kC1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;
  constexpr double kC2 = 0x1.62e42ff0c52d6p-1 / 32;
  const double xd = static_cast<double>(x);
  const double kds = __fma_rn(kInvLn2N, xd, kShift);
  const uint64_t ki = static_cast<uint64_t>(__double_as_longlong(kds));
  const double kd = __dsub_rn(kds, kShift);
  const double r = __fma_rn(kInvLn2N, xd, -kd);
  const uint64_t t = __ldg(&kExpfTab[ki & 31u]) + (ki << 47);
  const double s = __longlong_as_double(static_cast<long long>(t));
  const double z = __fma_rn(kC0, r, kC1);
  const double r2 = __dmul_rn(r, r);
  const double y = __fma_rn(z, r2, __fma_rn(kC2, r, 1.0));
  return __double2float_rn(__dmul_rn(y, s));
}

// x / (1 + exp(-x)) with the reference's +-20 cut-offs (silu.rs:47-61), exp as the host libm's.
// A NaN input comes back as itself, quieted: the host's division returns its first operand's
// NaN, while the device's would return the canonical NaN.
__device__ __forceinline__ float act_silu(float x) {
  if (x != x) return __uint_as_float(__float_as_uint(x) | 0x00400000u);
  if (x > 20.0f) return x;
  if (x < -20.0f) return 0.0f;
  return __fdiv_rn(x, __fadd_rn(1.0f, expf_libm(-x)));
}

// RN(x / c) for the constants c = 3, 5, 7 and |x| < 2^17, without a division: q = RN(x * z),
// r = x - q*c (exact by FMA), RN(q + r*z), z = RN(1/c) -- the method for a divisor known in
// advance of Brisebarre, Muller and Raina (IEEE Trans. Computers 53(8), 2004).  Checked
// exhaustively against IEEE division for every float below 2^17 in magnitude: identical
// except that x = -0 gives +0, which leaves the GELU series below unchanged.
__device__ __forceinline__ float div_by_const(float x, float c, float z) {
  const float q = __fmul_rn(x, z);
  return __fmaf_rn(__fmaf_rn(-q, c, x), z, q);
}

// The reference's tanh for GELU: the odd series x - x^3/3 + x^5/5 - x^7/7 below |x| <= 5,
// +-1 beyond (gelu.rs:91-103), evaluated in its order with correctly rounded division
// (|x^7| <= 78125 < 2^17 on this branch).
__device__ __forceinline__ float gelu_tanh_poly(float x) {
  if (x > 5.0f) return 1.0f;
  if (x < -5.0f) return -1.0f;
  constexpr float kInv3 = 1.0f / 3.0f, kInv5 = 1.0f / 5.0f, kInv7 = 1.0f / 7.0f;
  const float x2 = __fmul_rn(x, x);
  const float x3 = __fmul_rn(x2, x);
  const float x5 = __fmul_rn(x3, x2);
  const float x7 = __fmul_rn(x5, x2);
  float r = __fsub_rn(x, div_by_const(x3, 3.0f, kInv3));
  r = __fadd_rn(r, div_by_const(x5, 5.0f, kInv5));
  return __fsub_rn(r, div_by_const(x7, 7.0f, kInv7));
}

// Gelu::tanh_gelu (gelu.rs:77-85): 0.5 * x * (1 + tanh(sqrt(2/pi) * (x + 0.044715 * x^3))).
__device__ __forceinline__ float act_gelu(float x) {
  const float x_cube = __fmul_rn(__fmul_rn(x, x), x);
  const float arg = __fmul_rn(0.7978845608f, __fadd_rn(x, __fmul_rn(0.044715f, x_cube)));
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, gelu_tanh_poly(arg)));
}

template <int ACT>
__device__ __forceinline__ float apply_act(float x) {
  if constexpr (ACT == LSC_ACT_RELU) return act_relu(x);
  else if constexpr (ACT == LSC_ACT_RELU6) return act_relu6(x);
  else if constexpr (ACT == LSC_ACT_SILU) return act_silu(x);
  else if constexpr (ACT == LSC_ACT_GELU) return act_gelu(x);
  else return x;
}

// R(t) then Rust's clamp(-128,127) `as i8`: NaN -> 0.
template <int RND>
__device__ __forceinline__ int32_t requant_i8(float y, float s_out) {
  const float t = __fdiv_rn(y, s_out);
  float r = (RND == LSC_ROUND_HALF_EVEN) ? rintf(t) : roundf(t);
  if (r != r) return 0;
  if (r < -128.0f) r = -128.0f;
  if (r > 127.0f) r = 127.0f;
  return __float2int_rz(r);
}

// max that returns NaN when either operand is NaN (fmaxf returns the other one).
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// a and b saturated to int8 and packed: b in bits 7:0, a in bits 15:8, c's low 16 bits in
// bits 31:16.
__device__ __forceinline__ uint32_t pack_sat_s8(int32_t a, int32_t b, uint32_t c) {
  uint32_t d;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// two-lane f32 arithmetic (sm_100): each op rounds both lanes to nearest like its scalar form
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// act_gelu on two values with two-lane arithmetic: the same operations in the same order, so
// bit-identical to the scalar form.  The series is evaluated for every argument and replaced
// by +-1 beyond |t| > 5 afterwards (an overflowed series there is discarded).
// x + 0.044715 * x^3 is computed with scalar intrinsics: ptxas contracts a mul.rn.f32x2 whose
// only use is an add.rn.f32x2 into a single fma.rn.f32x2 (one rounding where the reference
// rounds twice), and the scalar .rn forms are never contracted.
__device__ __forceinline__ void act_gelu2(float& a, float& b) {
  const uint64_t x = f2pack(a, b);
  const uint64_t x_cube = f2mul(f2mul(x, x), x);
  float ca, cb;
  f2unpack(x_cube, ca, cb);
  const uint64_t inner = f2pack(__fadd_rn(a, __fmul_rn(0.044715f, ca)), __fadd_rn(b, __fmul_rn(0.044715f, cb)));
  const uint64_t t = f2mul(f2pack(0.7978845608f, 0.7978845608f), inner);
  const uint64_t t2 = f2mul(t, t);
  const uint64_t t3 = f2mul(t2, t);
  const uint64_t t5 = f2mul(t3, t2);
  const uint64_t t7 = f2mul(t5, t2);
  // x / c as div_by_const: q = x*z, r = fma(q, -c, x), fma(r, z, q)
  auto div2 = [](uint64_t v, float c, float z) {
    const uint64_t z2 = f2pack(z, z);
    const uint64_t q = f2mul(v, z2);
    return f2fma(f2fma(q, f2pack(-c, -c), v), z2, q);
  };
  uint64_t r = f2sub(t, div2(t3, 3.0f, 1.0f / 3.0f));
  r = f2add(r, div2(t5, 5.0f, 1.0f / 5.0f));
  r = f2sub(r, div2(t7, 7.0f, 1.0f / 7.0f));
  float ta, tb, ra, rb;
  f2unpack(t, ta, tb);
  f2unpack(r, ra, rb);
  ra = ta > 5.0f ? 1.0f : (ta < -5.0f ? -1.0f : ra);
  rb = tb > 5.0f ? 1.0f : (tb < -5.0f ? -1.0f : rb);
  const uint64_t y = f2mul(f2mul(f2pack(0.5f, 0.5f), x), f2add(f2pack(1.0f, 1.0f), f2pack(ra, rb)));
  f2unpack(y, a, b);
}

// requant_i8 for W values, packed four to a word (value j in byte j%4 of pk[j/4]), without
// the per-element IEEE division; same results.
//
// t = RN(y * inv_s) with inv_s = RN(1 / s_out) differs from the correctly rounded quotient
// RN(y / s_out) by at most 1.5 * 2^-23 * |t| (to first order).  t is clamped below at `lo`
// (-256, or 0 when a ReLU is folded in: with s_out > 0, R(max(y, 0) / s_out) =
// max(R(y / s_out), 0)), and adding 1.5 * 2^23 rounds it to an integer held in the float's
// low mantissa bits; the float stays positive, so its bit pattern minus that of 1.5 * 2^23 is
// an integer ordered like t (exactly rint(t) while t < 2^22) and the saturating pack clamps
// it to [-128, 127].  d = tc - rint(tc) is the distance to that integer, so 0.5 - |d| is the
// distance to the nearest half-integer; when RN(|d| + |tc| * 2^-22) < 0.5 (round-to-nearest
// is monotonic, so the unrounded sum is below 0.5 too) that distance exceeds the error above,
// the correctly rounded quotient lies strictly on the same side of the half-integer, and it
// rounds to the same integer in either rounding mode (the modes differ only at exact ties).
// The other elements -- near a half-integer, |t| >= 2^21, NaN (kept by the NaN-propagating
// clamp) -- are redone with the division: on random data a few in 10^5.  inv_s = 0 marks an
// s_out without a normal reciprocal: then every element takes the division.  A ReLU is
// folded only with s_out > 0.
template <int W, int RND>
__device__ __forceinline__ void requant_pack_rnd(const float (&y)[W], float s_out, float inv_s,
                                                 bool relu_folded, uint32_t (&pk)[W / 4]) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  constexpr int32_t kMagicBits = 0x4B400000;
  constexpr float kErr = 2.384185791015625e-7f;  // 2^-22
  const float lo = relu_folded ? 0.0f : -256.0f;
  bool slow = inv_s == 0.0f;
  const uint64_t inv2 = f2pack(inv_s, inv_s), mag2 = f2pack(kMagic, kMagic);
#pragma unroll
  for (int w = 0; w < W / 4; ++w) {
    int32_t v[4];
#pragma unroll
    for (int t = 0; t < 4; t += 2) {
      float t0, t1;
      f2unpack(f2mul(f2pack(y[4 * w + t], y[4 * w + t + 1]), inv2), t0, t1);
      const float c0 = fmax_nan(t0, lo), c1 = fmax_nan(t1, lo);
      const uint64_t tc2 = f2pack(c0, c1);
      const uint64_t tm2 = f2add(tc2, mag2);
      float d0, d1, m0, m1;
      f2unpack(f2sub(tc2, f2sub(tm2, mag2)), d0, d1);
      f2unpack(tm2, m0, m1);
      slow |= !(__fmaf_rn(fabsf(c0), kErr, fabsf(d0)) < 0.5f);
      slow |= !(__fmaf_rn(fabsf(c1), kErr, fabsf(d1)) < 0.5f);
      v[t] = __float_as_int(m0) - kMagicBits;
      v[t + 1] = __float_as_int(m1) - kMagicBits;
    }
    pk[w] = pack_sat_s8(v[1], v[0], pack_sat_s8(v[3], v[2], 0u));
  }
  if (__builtin_expect(slow, 0)) {
    const bool all = inv_s == 0.0f;
#pragma unroll
    for (int j = 0; j < W; ++j) {
      const float tc = fmax_nan(__fmul_rn(y[j], inv_s), lo);
      const float d = __fsub_rn(tc, __fsub_rn(__fadd_rn(tc, kMagic), kMagic));
      if (all || !(__fmaf_rn(fabsf(tc), kErr, fabsf(d)) < 0.5f)) {
        const float yj = relu_folded ? act_relu(y[j]) : y[j];
        const uint32_t q = static_cast<uint32_t>(requant_i8<RND>(yj, s_out)) & 0xFFu;
        const int sh = 8 * (j & 3);
        pk[j >> 2] = (pk[j >> 2] & ~(0xFFu << sh)) | (q << sh);
      }
    }
  }
}

// One value of requant_pack_rnd: the same reciprocal form and exactness test, with the
// division taken inline when the test fails.  Returns the int8 code in [-128, 127].
template <int RND>
__device__ __forceinline__ int32_t requant_one(float y, float s_out, float inv_s) {
  constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
  constexpr int32_t kMagicBits = 0x4B400000;
  constexpr float kErr = 2.384185791015625e-7f;  // 2^-22
  const float tc = fmax_nan(__fmul_rn(y, inv_s), -256.0f);
  const float tm = __fadd_rn(tc, kMagic);
  const float d = __fsub_rn(tc, __fsub_rn(tm, kMagic));
  if (inv_s != 0.0f && __fmaf_rn(fabsf(tc), kErr, fabsf(d)) < 0.5f) {
    const int32_t v = __float_as_int(tm) - kMagicBits;
    return v < -128 ? -128 : (v > 127 ? 127 : v);
  }
  return requant_i8<RND>(y, s_out);
}

template <int W>
__device__ __forceinline__ void requant_pack(const float (&y)[W], float s_out, float inv_s,
                                             bool relu_folded, int rounding, uint32_t (&pk)[W / 4]) {
  if (rounding == LSC_ROUND_HALF_EVEN) requant_pack_rnd<W, LSC_ROUND_HALF_EVEN>(y, s_out, inv_s, relu_folded, pk);
  else requant_pack_rnd<W, LSC_ROUND_HALF_AWAY>(y, s_out, inv_s, relu_folded, pk);
}


}  // namespace lsc
