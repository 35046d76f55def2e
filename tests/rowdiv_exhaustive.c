/* Exhaustive check of the rowwise quantisers' quotient (e4m3_quotient in
 * fastforward_b200/csrc/common.cuh) against the IEEE divide it replaces.
 *
 * Domain: every non-negative finite bf16 a (the row's largest |x|), s = max(a, 1e-12) / 448
 * (IEEE divide), r = 1 / s (IEEE, correctly rounded), and every bf16 x with |x| <= a, both
 * signs.  For each pair the e4m3 byte (round to nearest even, saturating at 448, sign kept)
 * of clamp(x / s, +-448) must equal that of clamp(q, +-448) with
 *     q0 = x r,  q = q0 + (x - q0 s) r  (both fused multiply-adds),  q |= sign(x).
 * Compiled with -ffp-contract=off, so every operation is one IEEE-rounded operation as on
 * the GPU (__fmul_rn, __fmaf_rn, __frcp_rn, __fdiv_rn).  Prints the counts; exits 1 on any
 * byte mismatch.  This file is test infrastructure only. */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>

static double e4m3_val[127]; /* value of the positive codes 0x00 .. 0x7e */

static float bf16(uint32_t bits) {
  const uint32_t u = bits << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* e4m3 (fn) byte of v: round to nearest, ties to the even code, saturate at 448. */
static int e4m3_byte(float v) {
  const int sign = signbit(v) ? 0x80 : 0;
  const double m = fabs((double)v);
  if (m >= 448.0) return sign | 0x7e;
  int lo = 0, hi = 126;
  while (hi - lo > 1) {
    const int mid = (lo + hi) / 2;
    if (e4m3_val[mid] <= m) lo = mid;
    else hi = mid;
  }
  const double dl = m - e4m3_val[lo], dh = e4m3_val[hi] - m;
  const int c = dl < dh ? lo : (dh < dl ? hi : ((lo & 1) ? hi : lo));
  return sign | c;
}

static float clamp448(float v) { return fminf(448.f, fmaxf(-448.f, v)); }

static float corrected_quotient(float x, float s, float r) {
  const float q0 = x * r;
  float q = fmaf(fmaf(-q0, s, x), r, q0);
  uint32_t qi, xi;
  memcpy(&qi, &q, 4);
  memcpy(&xi, &x, 4);
  qi |= xi & 0x80000000u;
  memcpy(&q, &qi, 4);
  return q;
}

int main(void) {
  for (int c = 0; c < 127; ++c) {
    const int e = c >> 3, m = c & 7;
    e4m3_val[c] = e == 0 ? ldexp(m / 8.0, -6) : ldexp(1.0 + m / 8.0, e - 7);
  }
  long long pairs = 0, fp32_diff = 0, byte_diff = 0;
#pragma omp parallel for schedule(dynamic, 64) reduction(+ : pairs, fp32_diff, byte_diff)
  for (int ab = 0; ab < 0x7f80; ++ab) { /* every non-negative finite bf16 */
    const float a = bf16((uint32_t)ab);
    const float s = fmaxf(a, 1e-12f) / 448.f;
    const float r = 1.0f / s;
    for (int xb = 0; xb <= ab; ++xb)
      for (int neg = 0; neg < 2; ++neg) {
        const float x = bf16((uint32_t)xb | ((uint32_t)neg << 15));
        const float qe = x / s, qf = corrected_quotient(x, s, r);
        ++pairs;
        if (memcmp(&qe, &qf, 4) != 0) {
          ++fp32_diff;
          if (e4m3_byte(clamp448(qe)) != e4m3_byte(clamp448(qf))) ++byte_diff;
        }
      }
  }
  printf("pairs %lld fp32_differs %lld byte_differs %lld\n", pairs, fp32_diff, byte_diff);
  return byte_diff != 0;
}
