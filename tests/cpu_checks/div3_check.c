/* Exhaustive check of the epilogues' division by three (prime-tts_b200/csrc/ptx.cuh, div3_rn):
 * q = RN(x * RN(1/3)), e = x - 3q computed exactly by one fused multiply-add, result q when e is
 * zero or x is infinite, else RN(q + e * RN(1/3)) -- against the IEEE quotient x / 3 for every
 * fp32 bit pattern.  Prints the number of mismatches (NaN inputs count as equal when both results
 * are NaN). */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

static float div3_rn(float x) {
  const float r = 0.3333333432674407958984375f;
  const float q = x * r;
  const float e = fmaf(-q, 3.0f, x);
  return (e == 0.0f || isinf(x)) ? q : fmaf(e, r, q);
}

int main(void) {
  unsigned long long bad = 0;
#pragma omp parallel for reduction(+ : bad) schedule(static)
  for (long long hi = 0; hi < 65536; ++hi) {
    for (uint32_t lo = 0; lo < 65536; ++lo) {
      const uint32_t b = ((uint32_t)hi << 16) | lo;
      float x;
      memcpy(&x, &b, 4);
      volatile float ref = x / 3.0f;
      const float got = div3_rn(x);
      float rr = ref;
      uint32_t a1, a2;
      memcpy(&a1, &rr, 4);
      memcpy(&a2, &got, 4);
      if (a1 != a2 && !(isnan(rr) && isnan(got))) ++bad;
    }
  }
  printf("%llu\n", bad);
  return 0;
}
