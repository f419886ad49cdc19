/* Checks the GELU epilogue's division by the constants 3, 5 and 7 (q = RN(x*z),
 * r = fma(-q, c, x), RN(fma(r, z, q)), z = RN(1/c)) against IEEE division, x86 SSE division
 * and fmaf being correctly rounded.  Arguments: lo hi -- the range of float bit patterns
 * [lo, hi) checked, for x and -x.  Prints the number of mismatches per divisor (zero results
 * are compared by value, so -0 against +0 is no mismatch) and exits non-zero if any. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float from_bits(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

static int same(float a, float b) {
  uint32_t ua, ub;
  memcpy(&ua, &a, 4);
  memcpy(&ub, &b, 4);
  return ua == ub || (a == 0.0f && b == 0.0f);
}

int main(int argc, char** argv) {
  if (argc < 3) return 2;
  const uint32_t lo = (uint32_t)strtoul(argv[1], NULL, 0), hi = (uint32_t)strtoul(argv[2], NULL, 0);
  const float cs[3] = {3.0f, 5.0f, 7.0f};
  long long total_bad = 0;
  for (int k = 0; k < 3; ++k) {
    const volatile float c = cs[k];
    const float z = 1.0f / c;
    long long bad = 0;
#pragma omp parallel for reduction(+ : bad) schedule(static)
    for (long long uu = lo; uu < (long long)hi; ++uu) {
      const uint32_t u = (uint32_t)uu;
      for (int sgn = 0; sgn < 2; ++sgn) {
        const float x = sgn ? -from_bits(u) : from_bits(u);
        const float q = x * z;
        const float got = fmaf(fmaf(-q, c, x), z, q);
        if (!same(got, x / c)) ++bad;
      }
    }
    printf("c=%g bad=%lld\n", (double)cs[k], bad);
    total_bad += bad;
  }
  return total_bad ? 1 : 0;
}
