// Row kernels of the vision tower in front of the language path: LayerNorm (the blocks'
// norm1 / norm2 and the mergers' norms) and the 2-D vision rotary applied to the qkv
// projection, which also lays q, k and v out head-major for the attention kernel.
//
// Replace, in the reference's vision wrappers: the LayerNorm modules of the HF blocks and
// mergers (_legacy/vision_graph_runtime.py:16-27, `VisionGraph.core`; the fused add +
// LayerNorm of _legacy/lower_kernels.py:115-136 is the residual add, which the producing
// GEMM's epilogue does here) and `_vision_rope` (_legacy/search_kernels.py:111-125).
#include "common.cuh"
#include "pdl.cuh"

namespace {

__device__ __forceinline__ void unpack8(uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// One CTA per row, C / 8 threads (rounded up to whole warps) of 8 consecutive elements.
// mean and variance from float64 sums of x and x^2 (exact for bf16 inputs of the usual
// range, so independent of the reduction order): mean = fp32(S1 / C),
// rstd = fp32(1 / sqrt(max(S2 / C - (S1 / C)^2, 0) + eps)) in IEEE float64 operations;
// y = bf16(((x - mean) * rstd) * w + b) in IEEE fp32 operations in that order.
// With add != NULL the row is first x = bf16(x + add) (the residual add of the reference's
// add + LayerNorm), written to `residual`.
__global__ void __launch_bounds__(1024) layernorm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ add,
                                                         const uint16_t* __restrict__ w, const uint16_t* __restrict__ b,
                                                         float eps, uint16_t* residual, uint16_t* y, int C) {
  pdl_wait();
  pdl_launch();
  __shared__ double red[2][32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = blockDim.x >> 5;
  const size_t off = (size_t)blockIdx.x * C + (size_t)tid * 8;
  const bool active = tid * 8 < C;  // the block is rounded up to whole warps
  float f[8];
  unpack8(active ? *reinterpret_cast<const uint4*>(x + off) : make_uint4(0, 0, 0, 0), f);
  if (add != nullptr && active) {
    float g[8];
    unpack8(*reinterpret_cast<const uint4*>(add + off), g);
    uint32_t r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = round_bf(__fadd_rn(f[2 * i], g[2 * i]));
      f[2 * i + 1] = round_bf(__fadd_rn(f[2 * i + 1], g[2 * i + 1]));
      r[i] = (uint32_t)f2bf(f[2 * i]) | ((uint32_t)f2bf(f[2 * i + 1]) << 16);
    }
    *reinterpret_cast<uint4*>(residual + off) = make_uint4(r[0], r[1], r[2], r[3]);
  }
  double s1 = 0.0, s2 = 0.0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s1 = __dadd_rn(s1, (double)f[i]);
    s2 = __dadd_rn(s2, __dmul_rn((double)f[i], (double)f[i]));
  }
  s1 = warp_sum_d(s1);
  s2 = warp_sum_d(s2);
  if (lane == 0) {
    red[0][warp] = s1;
    red[1][warp] = s2;
  }
  __syncthreads();
  if (warp == 0) {
    double a = lane < nw ? red[0][lane] : 0.0, c = lane < nw ? red[1][lane] : 0.0;
    a = warp_sum_d(a);
    c = warp_sum_d(c);
    if (lane == 0) {
      red[0][0] = a;
      red[1][0] = c;
    }
  }
  __syncthreads();
  const double mean_d = __ddiv_rn(red[0][0], (double)C);
  double var_d = __dsub_rn(__ddiv_rn(red[1][0], (double)C), __dmul_rn(mean_d, mean_d));
  if (var_d < 0.0) var_d = 0.0;
  const float mean = (float)mean_d;
  const float rstd = (float)__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(var_d, (double)eps)));
  if (!active) return;
  float wv[8], bv[8];
  unpack8(__ldg(reinterpret_cast<const uint4*>(w + tid * 8)), wv);
  unpack8(__ldg(reinterpret_cast<const uint4*>(b + tid * 8)), bv);
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float r[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int e = 2 * i + j;
      r[j] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(f[e], mean), rstd), wv[e]), bv[e]);
    }
    o[i] = (uint32_t)f2bf(r[0]) | ((uint32_t)f2bf(r[1]) << 16);
  }
  *reinterpret_cast<uint4*>(y + off) = make_uint4(o[0], o[1], o[2], o[3]);
}

// One CTA per patch, one thread per 8 columns of a head of q, k or v: the patch's qkv row
// (and its cos / sin rows) staged in shared memory with 16-byte loads, then each thread
// writes 16 bytes of the head-major output.  qkv row p = [q (H x d) | k (H x d) |
// v (H x d)]; cos / sin [P, d] fp32.  q, k: y[c] = x[c] cos[c] + r[c] sin[c] with
// r = (-x[c + d/2] for c < d/2, x[c - d/2] otherwise), both products and the sum IEEE fp32
// operations, then bf16; v copied.  Outputs [H, P, dp]: columns [0, d) written, columns
// [d, dp) (the attention kernel's zero padding) left as they are.
__global__ void vision_rope_kernel(const uint16_t* __restrict__ qkv, const float* __restrict__ cs,
                                   const float* __restrict__ sn, int P, int H, int d, int dp, uint16_t* q,
                                   uint16_t* k, uint16_t* v) {
  extern __shared__ __align__(16) uint8_t vr_smem[];
  const int hd = H * d;
  uint16_t* srow = reinterpret_cast<uint16_t*>(vr_smem);                             // [3 * H * d]
  float* scos = reinterpret_cast<float*>(vr_smem + ((size_t)3 * hd * 2 + 15) / 16 * 16);  // [d]
  float* ssin = scos + d;                                                               // [d]
  pdl_wait();
  pdl_launch();
  const int p = blockIdx.x, half = d / 2;
  const uint16_t* src = qkv + (size_t)p * 3 * hd;
  for (int i = threadIdx.x; i < 3 * hd / 8; i += blockDim.x)
    reinterpret_cast<uint4*>(srow)[i] = reinterpret_cast<const uint4*>(src)[i];
  for (int i = threadIdx.x; i < d / 4; i += blockDim.x) {  // d is a multiple of 8
    reinterpret_cast<float4*>(scos)[i] = __ldg(reinterpret_cast<const float4*>(cs + (size_t)p * d) + i);
    reinterpret_cast<float4*>(ssin)[i] = __ldg(reinterpret_cast<const float4*>(sn + (size_t)p * d) + i);
  }
  __syncthreads();
  const int cpr = d / 8;  // 16-byte chunks per head row
  for (int t = threadIdx.x; t < 3 * H * cpr; t += blockDim.x) {
    const int part = t / (H * cpr), rem = t - part * H * cpr, h = rem / cpr, c0 = (rem - h * cpr) * 8;
    const uint16_t* row = srow + (size_t)part * hd + h * d;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float y[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int c = c0 + 2 * e + j;
        const float xv = bf2f(row[c]);
        if (part == 2) {
          y[j] = xv;
        } else {
          const float rv = c < half ? -bf2f(row[c + half]) : bf2f(row[c - half]);
          y[j] = __fadd_rn(__fmul_rn(xv, scos[c]), __fmul_rn(rv, ssin[c]));
        }
      }
      w[e] = (uint32_t)f2bf(y[0]) | ((uint32_t)f2bf(y[1]) << 16);
    }
    uint16_t* dst = part == 0 ? q : (part == 1 ? k : v);
    *reinterpret_cast<uint4*>(dst + ((size_t)h * P + p) * dp + c0) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

}  // namespace

extern "C" int ffb_add_layernorm(const uint16_t* a, const uint16_t* add, const uint16_t* w, const uint16_t* b,
                                 float eps, uint16_t* residual, uint16_t* y, int rows, int C, void* stream) {
  FFB_REQUIRE(a && w && b && y, "ffb_layernorm: NULL pointer");
  FFB_REQUIRE(!add || residual, "ffb_add_layernorm: the sum needs a residual output");
  FFB_REQUIRE(rows > 0 && C >= 8 && C % 8 == 0 && C <= 8192, "ffb_layernorm: rows=%d C=%d (C a multiple of 8, <= 8192)",
              rows, C);
  FFB_REQUIRE(ffb::aligned(a, 16) && ffb::aligned(w, 16) && ffb::aligned(b, 16) && ffb::aligned(y, 16) &&
                  (!add || ffb::aligned(add, 16)) && (!residual || ffb::aligned(residual, 16)),
              "ffb_layernorm: pointers must be 16-byte aligned");
  const int threads = (C / 8 + 31) / 32 * 32;
  cudaError_t e = ffb::launch(layernorm_kernel, dim3(rows), dim3(threads), 0, (cudaStream_t)stream, a, add, w, b, eps,
                              residual, y, C);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_layernorm: launch: %s", cudaGetErrorString(e));
  return FFB_OK;
}

extern "C" int ffb_layernorm(const uint16_t* x, const uint16_t* w, const uint16_t* b, float eps, uint16_t* y, int rows,
                             int C, void* stream) {
  return ffb_add_layernorm(x, nullptr, w, b, eps, nullptr, y, rows, C, stream);
}

extern "C" int ffb_vision_rope(const uint16_t* qkv, const float* cos, const float* sin, int P, int H, int d, int dp,
                               uint16_t* q, uint16_t* k, uint16_t* v, void* stream) {
  FFB_REQUIRE(qkv && cos && sin && q && k && v, "ffb_vision_rope: NULL pointer");
  FFB_REQUIRE(P > 0 && H > 0 && d > 0 && d % 8 == 0 && dp >= d && dp % 8 == 0 && dp <= 256 && H * d <= 7680,
              "ffb_vision_rope: bad shape P=%d H=%d d=%d dp=%d (d, dp multiples of 8)", P, H, d, dp);
  FFB_REQUIRE(ffb::aligned(qkv, 16) && ffb::aligned(q, 16) && ffb::aligned(k, 16) && ffb::aligned(v, 16),
              "ffb_vision_rope: qkv, q, k, v must be 16-byte aligned");
  const int work = 3 * H * (d / 8);
  const int threads = work < 1024 ? (work + 31) / 32 * 32 : 1024;
  FFB_REQUIRE(ffb::aligned(cos, 16) && ffb::aligned(sin, 16), "ffb_vision_rope: cos and sin must be 16-byte aligned");
  const size_t smem = ((size_t)3 * H * d * 2 + 15) / 16 * 16 + (size_t)2 * d * 4;
  cudaError_t e = ffb::launch(vision_rope_kernel, dim3(P), dim3(threads), smem, (cudaStream_t)stream, qkv, cos, sin, P,
                              H, d, dp, q, k, v);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_vision_rope: launch: %s", cudaGetErrorString(e));
  return FFB_OK;
}
