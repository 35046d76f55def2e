/*
 * attn.c - CPU restatement of the arithmetic of the causal attention kernel's online
 * softmax (TEST INFRASTRUCTURE ONLY: the oracle links it, the product never does).
 *
 * The reference's kernel (_legacy/limit_kernels.py:8-33) fixes the algorithm: fp32 scores
 * scaled by 1/sqrt(128), an online softmax over 64-key blocks with running max m and
 * denominator l, alpha = exp(m_old - m_new), P cast to bf16 before P.V, output
 * bf16(acc / l).  It leaves the exponential (tl.exp) and the reduction orders to the
 * compiler.  The CUDA kernel fixes both, and these functions restate them operation for
 * operation, so that the two agree bit for bit:
 *   x = fp32(s * scale_log2) (masked keys -inf); block max over the 64 keys;
 *   m_new = max(m, block max); base = m_new (0 while the row has seen no key);
 *   alpha = exp2_poly(m - base); p = exp2_poly(x - base);
 *   four parts of 16 keys each keep their own denominator share:
 *     psum = sum over the part's 8 key pairs of (p0 + p1), in key order,
 *     l_part = fma(l_part, alpha, psum);
 *   o = fma(o, alpha, O_j) per output column, O_j = P_j . V_j on the tensor core;
 *   l = ((l_0 + l_1) + l_2) + l_3; out = bf16(fp32(o / l)) (IEEE quotient).
 * exp2_poly is this project's own exponential: 2^x = 2^n * 2^f with n = rint(x),
 * f = x - n in [-1/2, 1/2], and 2^f by the degree-7 Taylor polynomial of e^(f ln 2)
 * (coefficients (ln 2)^k / k!, rounded to fp32) in Horner form with fused multiply-adds;
 * results below 2^-125 are 0.  It is within a few fp32 ulps of 2^x, far inside the bf16
 * rounding of P.
 *
 * Build: with tcgemm.c into oracle/_build/libtcgemm.so (make -C oracle).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static const float EXP2_C[8] = {
    1.0f,
    0.693147180559945309f,     /* ln 2 */
    0.240226506959100712f,     /* (ln 2)^2 / 2 */
    0.0555041086648215800f,    /* (ln 2)^3 / 6 */
    0.00961812910762847717f,   /* (ln 2)^4 / 24 */
    0.00133335581464284434f,   /* (ln 2)^5 / 120 */
    0.000154035303933816099f,  /* (ln 2)^6 / 720 */
    1.52527338040598403e-05f,  /* (ln 2)^7 / 5040 */
};

float ffo_exp2(float x) {
  if (!(x >= -125.0f)) return 0.0f; /* -inf, NaN and results below 2^-125 */
  const float n = rintf(x);         /* nearest, ties to even */
  const float f = x - n;            /* exact */
  float p = EXP2_C[7];
  for (int k = 6; k >= 0; --k) p = fmaf(p, f, EXP2_C[k]);
  uint32_t b;
  memcpy(&b, &p, 4);
  b += (uint32_t)((int32_t)n << 23); /* p * 2^n: p in [0.70, 1.42], result normal */
  float y;
  memcpy(&y, &b, 4);
  return y;
}

void ffo_exp2_array(const float* x, float* y, int n) {
  for (int i = 0; i < n; ++i) y[i] = ffo_exp2(x[i]);
}

static uint16_t bf16_rne(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40); /* NaN stays NaN */
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/*
 * One 64-key block of the online softmax for R rows.
 *   S      [R][64] fp32 raw scores (q . k accumulated on the tensor core) of keys
 *          key0 .. key0 + 63
 *   qpos   [R] each row's position (keys > qpos are masked), lo [R] its lowest visible key
 *   T      keys >= T are masked
 *   m      [R] running max (updated), l [R][4] denominator parts (updated)
 *   P      [R][64] bf16 out, alpha [R] out
 */
void attn_softmax_block(const float* S, int R, const int* qpos, const int* lo, int T, int key0, float scale_log2,
                        float* m, float* l, uint16_t* P, float* alpha) {
  for (int r = 0; r < R; ++r) {
    float x[64];
    float bmax = -INFINITY;
    for (int c = 0; c < 64; ++c) {
      const int key = key0 + c;
      const int masked = key > qpos[r] || key >= T || key < lo[r];
      x[c] = masked ? -INFINITY : S[(size_t)r * 64 + c] * scale_log2;
      bmax = fmaxf(bmax, x[c]);
    }
    const float nm = fmaxf(m[r], bmax);
    const float base = nm == -INFINITY ? 0.0f : nm;
    const float a = ffo_exp2(m[r] - base);
    m[r] = nm;
    alpha[r] = a;
    for (int part = 0; part < 4; ++part) {
      float psum = 0.0f;
      for (int c = 0; c < 2; ++c)
        for (int e = 0; e < 4; ++e) {
          const int k0 = 16 * part + 8 * c + 2 * e;
          const float p0 = ffo_exp2(x[k0] - base), p1 = ffo_exp2(x[k0 + 1] - base);
          psum = psum + (p0 + p1);
          P[(size_t)r * 64 + k0] = bf16_rne(p0);
          P[(size_t)r * 64 + k0 + 1] = bf16_rne(p1);
        }
      l[r * 4 + part] = fmaf(l[r * 4 + part], a, psum);
    }
  }
}

/* o[r][d] = fma(o[r][d], alpha[r], O[r][d]) over R rows of 128 columns. */
void attn_fold(float* o, const float* O, const float* alpha, int R) {
  for (int r = 0; r < R; ++r)
    for (int d = 0; d < 128; ++d) o[(size_t)r * 128 + d] = fmaf(o[(size_t)r * 128 + d], alpha[r], O[(size_t)r * 128 + d]);
}

/* out[r][d] = bf16(fp32(o / l)) with l = ((l0 + l1) + l2) + l3. */
void attn_finish(const float* o, const float* l, int R, uint16_t* out) {
  for (int r = 0; r < R; ++r) {
    const float den = ((l[r * 4] + l[r * 4 + 1]) + l[r * 4 + 2]) + l[r * 4 + 3];
    for (int d = 0; d < 128; ++d) out[(size_t)r * 128 + d] = bf16_rne(o[(size_t)r * 128 + d] / den);
  }
}
