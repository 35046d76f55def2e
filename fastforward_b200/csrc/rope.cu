// Per-head QK RMSNorm + rotate-half RoPE with the interleaved M-RoPE cos/sin tables,
// writing Q/K (and a V copy) head-major for the attention kernel.
//
// Reference rounding (_legacy/lower_kernels.py:66-86, `_rope_rows`), per (token, head):
//   inv = 1/sqrt(sum(x^2)/128 + eps) (exact float64 sum, IEEE sqrt/divide);
//   xn = bf16(bf16(x*inv)*w[i]);
//   rn  = bf16(bf16(x[i+-64]*inv)*w[i+-64]), negated for i < 64;
//   y   = bf16( bf16(xn*cos[t,i]) + bf16(rn*sin[t,i]) ).
// One warp per (token, head): lane l owns elements 4l..4l+3; the rotate-half partner
// (i +- 64) lives in lane l ^ 16, so the pair exchange is one shuffle.
#include "common.cuh"
#include "pdl.cuh"

namespace {

constexpr int D = 128;
constexpr int WARPS = 8;

struct RopeArgs {
  const uint16_t* qkv;
  const float* qkv32;
  int splits, row_stride;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  float eps;
  const uint16_t* cos;
  const uint16_t* sin;
  uint16_t* yq;
  uint16_t* yk;
  uint16_t* yv;
  int T, HQ, HK;
};

__device__ __forceinline__ void load4(const RopeArgs& p, int t, int col, float (&x)[4]) {
  if (p.qkv) {
    const uint2 u = *reinterpret_cast<const uint2*>(p.qkv + (size_t)t * p.row_stride + col);
    x[0] = __uint_as_float(u.x << 16);
    x[1] = __uint_as_float(u.x & 0xffff0000u);
    x[2] = __uint_as_float(u.y << 16);
    x[3] = __uint_as_float(u.y & 0xffff0000u);
  } else {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < p.splits; ++s) {
      const float4 v = *reinterpret_cast<const float4*>(p.qkv32 + ((size_t)s * p.T + t) * p.row_stride + col);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    x[0] = round_bf(acc.x); x[1] = round_bf(acc.y); x[2] = round_bf(acc.z); x[3] = round_bf(acc.w);
  }
}

__device__ __forceinline__ void store4(uint16_t* dst, const float (&y)[4]) {
  const uint32_t lo = (uint32_t)f2bf(y[0]) | ((uint32_t)f2bf(y[1]) << 16);
  const uint32_t hi = (uint32_t)f2bf(y[2]) | ((uint32_t)f2bf(y[3]) << 16);
  *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
}

__global__ void __launch_bounds__(WARPS * 32) qk_norm_rope_kernel(const RopeArgs p) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const int item = blockIdx.x * WARPS + (threadIdx.x >> 5);
  const int heads = p.HQ + 2 * p.HK;
  if (item >= p.T * heads) return;
  const int t = item / heads, h = item % heads;
  const int d0 = lane * 4;
  float x[4];
  load4(p, t, h * D + d0, x);
  if (h >= p.HQ + p.HK) {  // V head: copy
    if (p.yv) store4(p.yv + ((size_t)(h - p.HQ - p.HK) * p.T + t) * D + d0, x);
    return;
  }
  const bool is_q = h < p.HQ;
  const uint16_t* wn = is_q ? p.q_norm : p.k_norm;
  double ss = 0.0;
#pragma unroll
  for (int e = 0; e < 4; ++e) ss += (double)(x[e] * x[e]);
  const float inv = inv_rms_from_ss(warp_sum_d(ss), D, p.eps);
  float xn[4], rn[4], y[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) xn[e] = round_bf(round_bf(x[e] * inv) * bf2f(wn[d0 + e]));
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    rn[e] = __shfl_xor_sync(0xffffffffu, xn[e], 16);  // partner element i +- 64
    if (d0 < 64) rn[e] = -rn[e];
  }
  const uint16_t* c = p.cos + (size_t)t * D + d0;
  const uint16_t* s = p.sin + (size_t)t * D + d0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float left = round_bf(xn[e] * bf2f(c[e]));
    const float right = round_bf(rn[e] * bf2f(s[e]));
    y[e] = left + right;
  }
  uint16_t* dst = is_q ? p.yq + ((size_t)h * p.T + t) * D + d0 : p.yk + ((size_t)(h - p.HQ) * p.T + t) * D + d0;
  store4(dst, y);
}

}  // namespace

extern "C" int ffb_qk_norm_rope(const uint16_t* qkv, const float* qkv32, int splits, int row_stride,
                                const uint16_t* q_norm, const uint16_t* k_norm, float eps, const uint16_t* cos,
                                const uint16_t* sin, uint16_t* yq, uint16_t* yk, uint16_t* yv, int T, int HQ, int HK,
                                void* stream) {
  FFB_REQUIRE(qkv || (qkv32 && splits >= 1), "ffb_qk_norm_rope: need qkv or (qkv32, splits >= 1)");
  FFB_REQUIRE(q_norm && k_norm && cos && sin && yq && yk, "ffb_qk_norm_rope: NULL pointer");
  FFB_REQUIRE(T > 0 && HQ > 0 && HK > 0 && HQ % HK == 0, "ffb_qk_norm_rope: bad heads HQ=%d HK=%d", HQ, HK);
  FFB_REQUIRE(row_stride >= (HQ + 2 * HK) * D && row_stride % 4 == 0, "ffb_qk_norm_rope: row_stride %d", row_stride);
  FFB_REQUIRE((!qkv || ffb::aligned(qkv, 8)) && (!qkv32 || ffb::aligned(qkv32, 16)),
              "ffb_qk_norm_rope: input alignment");
  FFB_REQUIRE(ffb::aligned(yq, 8) && ffb::aligned(yk, 8) && (!yv || ffb::aligned(yv, 8)),
              "ffb_qk_norm_rope: output alignment");
  RopeArgs p = {qkv, qkv ? nullptr : qkv32, splits, row_stride, q_norm, k_norm, eps, cos, sin, yq, yk, yv, T, HQ, HK};
  const long long items = (long long)T * (HQ + 2 * HK);
  const int grid = (int)((items + WARPS - 1) / WARPS);
  cudaError_t e = ffb::launch(qk_norm_rope_kernel, dim3(grid), dim3(WARPS * 32), 0, (cudaStream_t)stream, p);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_qk_norm_rope: %s", cudaGetErrorString(e));
  return FFB_OK;
}
