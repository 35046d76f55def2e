/*
 * act.c - CPU restatement of the activations in the epilogue of the bf16 linear
 * (fastforward_b200/csrc/gemm_bf16.cu), operation for operation (TEST INFRASTRUCTURE ONLY).
 *
 * The vision tower's MLPs use GELU: tanh form in the blocks (`gelu_pytorch_tanh`), erf form
 * in the mergers (nn.GELU()).  Both are (x / 2) s, s = 1 + tanh(u) or 1 + erf(z), which the
 * kernel evaluates with IEEE-rounded fp32 operations, taking the small positive term itself
 * for negative arguments (no cancellation):
 *   tanh form: u = 0.7978845608 (x + 0.044715 ((x x) x)); r = 2 / (exp2_poly(|u| 2 log2 e) + 1)
 *     (0 for |u| >= 40); s = r for u < 0, else 2 - r; y = (0.5 x) s;
 *   erf form (Abramowitz & Stegun 7.1.26): z = x 0.7071067812, t = 1 / (1 + 0.3275911 |z|),
 *     p = t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) (Horner with fused multiply-adds),
 *     q = p exp2_poly((|z| |z|) (-log2 e)); s = q for z < 0, else 2 - q; y = (x 0.5) s.
 * ffo_exp2 (attn.c) is the same exponential the kernels use.
 */
#include <math.h>

float ffo_exp2(float x);

static float gelu_tanh(float x) {
  const float x3 = (x * x) * x;
  const float u = 0.797884560802865355f * (x + 0.044715f * x3);
  const float a = fabsf(u);
  float r = 0.0f;
  if (!(a >= 40.0f)) r = 2.0f / (ffo_exp2(a * 2.88539008177792681f) + 1.0f);
  const float s = u < 0.0f ? r : 2.0f - r;
  return (0.5f * x) * s;
}

static float gelu_erf(float x) {
  const float z = x * 0.707106781186547524f;
  const float a = fabsf(z);
  const float t = 1.0f / (1.0f + 0.3275911f * a);
  float p = 1.061405429f;
  p = fmaf(p, t, -1.453152027f);
  p = fmaf(p, t, 1.421413741f);
  p = fmaf(p, t, -0.284496736f);
  p = fmaf(p, t, 0.254829592f);
  p = p * t;
  const float q = p * ffo_exp2((a * a) * -1.44269504088896341f);
  const float s = z < 0.0f ? q : 2.0f - q;
  return (x * 0.5f) * s;
}

void ffo_gelu_tanh_array(const float* x, float* y, long n) {
  for (long i = 0; i < n; ++i) y[i] = gelu_tanh(x[i]);
}

void ffo_gelu_erf_array(const float* x, float* y, long n) {
  for (long i = 0; i < n; ++i) y[i] = gelu_erf(x[i]);
}
