/* The device's expf (lightship_b200/csrc/epilogue.cuh, expf_libm) restated in C with the
 * same double operations and fused multiply-adds, compared with this host's libm expf on
 * every float whose bits lie in [lo, hi).  Exit status 0 when all agree bit for bit.
 * Usage: expf_check <lo bits hex> <hi bits hex>  (e.g. 0xC1A00000 0xC1A00001 for one value) */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static const uint64_t kTab[32] = {
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull};

static float expf_restated(float x) {
  const double inv_ln2_n = 0x1.71547652b82fep+0 * 32, shift = 0x1.8p+52;
  const double c0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32, c1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;
  const double c2 = 0x1.62e42ff0c52d6p-1 / 32;
  const double xd = (double)x;
  const double kds = fma(inv_ln2_n, xd, shift);
  uint64_t ki;
  memcpy(&ki, &kds, 8);
  const double kd = kds - shift;
  const double r = fma(inv_ln2_n, xd, -kd);
  const uint64_t t = kTab[ki & 31u] + (ki << 47);
  double s;
  memcpy(&s, &t, 8);
  const double z = fma(c0, r, c1);
  const double y = fma(z, r * r, fma(c2, r, 1.0));
  return (float)(y * s);
}

int main(int argc, char** argv) {
  if (argc < 3) return 2;
  const uint64_t lo = strtoull(argv[1], 0, 16), hi = strtoull(argv[2], 0, 16);
  long bad = 0;
#pragma omp parallel for reduction(+ : bad) schedule(static, 1 << 16)
  for (int64_t u = (int64_t)lo; u < (int64_t)hi; ++u) {
    const uint32_t b = (uint32_t)u;
    float x;
    memcpy(&x, &b, 4);
    const float want = expf(x), got = expf_restated(x);
    uint32_t wb, gb;
    memcpy(&wb, &want, 4);
    memcpy(&gb, &got, 4);
    if (wb != gb) {
      if (bad < 5) printf("x=%a libm %a restated %a\n", x, want, got);
      ++bad;
    }
  }
  printf("%ld mismatches in [%#llx, %#llx)\n", bad, (unsigned long long)lo, (unsigned long long)hi);
  return bad != 0;
}
