/* Exhaustive check of the quantiser's division shortcut (test support, CPU only).
 *
 * For every E4M3 significand of the divisor d (1 + m/8, m = 0..7) and every FP32 significand of
 * the dividend x in [1, 2), with r = the correctly rounded 1/d:
 *     q1 = x*r;  rem = fma(-q1, d, x);  q = fma(rem, r, q1)
 * must equal the correctly rounded x/d bit for bit. Prints the mismatch count; exit status 0
 * when there are none. Built with -ffp-contract=off so each operation rounds once. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

static float bits_to_float(uint32_t u) {
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

static uint32_t float_to_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  return u;
}

int main(void) {
  long mismatches = 0;
  for (int m = 0; m < 8; ++m) {
    volatile float d = 1.0f + (float)m / 8.0f;
    volatile float one = 1.0f;
    const float r = one / d;
    for (uint32_t frac = 0; frac < (1u << 23); ++frac) {
      const float x = bits_to_float(0x3F800000u | frac);
      const float q1 = x * r;
      const float rem = fmaf(-q1, d, x);
      const float q = fmaf(rem, r, q1);
      if (float_to_bits(q) != float_to_bits(x / d)) ++mismatches;
    }
  }
  printf("%ld\n", mismatches);
  return mismatches != 0;
}
