// Small kernels at the two ends of the path: the embedding gather with the visual-row
// scatter, the standalone SwiGLU, and the tail readout (final add, final RMSNorm,
// option-row dots, log-softmax).
#include "common.cuh"
#include "pdl.cuh"

namespace {

constexpr int NT = 256;

// h[t] = visual[t - s] for s <= t < s + nv, else table[ids[t]]   (scaled_qwen_runtime.py:145)
__global__ void __launch_bounds__(NT) embed_kernel(const int64_t* __restrict__ ids, const uint16_t* __restrict__ table,
                                                   int64_t vocab, const uint16_t* __restrict__ visual, int s, int nv,
                                                   uint16_t* __restrict__ h, int H) {
  pdl_wait();
  pdl_launch();
  const int t = blockIdx.x;
  const uint16_t* src;
  if (visual && t >= s && t < s + nv) {
    src = visual + (size_t)(t - s) * H;
  } else {
    int64_t id = ids[t];
    if (id < 0 || id >= vocab) id = 0;  // host validates; a device-side clamp keeps reads in bounds
    src = table + (size_t)id * H;
  }
  uint16_t* dst = h + (size_t)t * H;
  for (int i = threadIdx.x; i < H / 8; i += NT)
    reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
}

// y = bf16(bf16(g / (1 + exp(-g))) * u)   (_legacy/search_kernels.py:8-15; exp = expf, IEEE divide)
__global__ void __launch_bounds__(NT) swiglu_kernel(const uint16_t* __restrict__ gate, const uint16_t* __restrict__ up,
                                                    int stride, uint16_t* __restrict__ y, int M, int I) {
  pdl_wait();
  pdl_launch();
  const size_t n = (size_t)M * I;
  for (size_t i = blockIdx.x * (size_t)NT + threadIdx.x; i < n; i += (size_t)gridDim.x * NT) {
    const size_t m = i / I, c = i % I;
    const float g = bf2f(gate[m * stride + c]);
    const float u = bf2f(up[m * stride + c]);
    const float act = round_bf(__fdiv_rn(g, 1.f + expf(-g)));
    y[i] = f2bf(act * u);
  }
}

__device__ __forceinline__ double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_d(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    double r = lane < NT / 32 ? red[lane] : 0.0;
    r = warp_sum_d(r);
    if (lane == 0) red[NT / 32] = r;
  }
  __syncthreads();
  const double r = red[NT / 32];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float r = lane < NT / 32 ? red[lane] : 0.f;
    r = warp_sum(r);
    if (lane == 0) red[NT / 32] = r;
  }
  __syncthreads();
  const float r = red[NT / 32];
  __syncthreads();
  return r;
}

// One CTA: chosen = bf16(res + mlp); xn = bf16(bf16(x*inv)*w); logits[o] = bf16(xn . head[o])
// (warp o computes option o); logprobs = log_softmax(logits[:k]).
// (_legacy/limit_kernels.py:48-57 + _family/night_runtime.py:104-105)
__global__ void __launch_bounds__(NT) readout_kernel(const uint16_t* __restrict__ res, const uint16_t* __restrict__ mlp,
                                                     const float* __restrict__ mlp32, int splits,
                                                     const uint16_t* __restrict__ w, float eps,
                                                     const uint16_t* __restrict__ head, int n, int k,
                                                     float* __restrict__ logits, float* __restrict__ logprobs, int H) {
  __shared__ double redd[NT / 32 + 1];
  __shared__ float z[8];
  extern __shared__ float xn[];  // H floats
  pdl_wait();
  pdl_launch();
  double ss = 0.0;
  for (int i = threadIdx.x; i < H; i += NT) {
    float x = bf2f(res[i]);
    if (mlp) {
      x = round_bf(x + bf2f(mlp[i]));
    } else if (mlp32) {
      float b = 0.f;
      for (int s = 0; s < splits; ++s) b += mlp32[(size_t)s * H + i];
      x = round_bf(x + round_bf(b));
    }
    xn[i] = x;
    ss += (double)(x * x);
  }
  const float inv = inv_rms_from_ss(block_sum_d(ss, redd), H, eps);
  for (int i = threadIdx.x; i < H; i += NT) xn[i] = round_bf(round_bf(xn[i] * inv) * bf2f(w[i]));
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp < n) {
    // bf16 x bf16 products are exact in fp32; their float64 sum is (nearly always) exact,
    // so the bf16-rounded logit does not depend on the reduction order
    const uint16_t* hr = head + (size_t)warp * H;
    double d = 0.0;
    for (int i = lane; i < H; i += 32) d += (double)(xn[i] * bf2f(hr[i]));
    d = warp_sum_d(d);
    if (lane == 0) {
      z[warp] = round_bf((float)d);
      logits[warp] = z[warp];
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && logprobs) {
    float m = -INFINITY;
    for (int i = 0; i < k; ++i) m = fmaxf(m, z[i]);
    float s = 0.f;
    for (int i = 0; i < k; ++i) s += expf(z[i] - m);
    const float lse = logf(s);
    for (int i = 0; i < k; ++i) logprobs[i] = z[i] - m - lse;
  }
}

}  // namespace

extern "C" int ffb_embed_gather(const int64_t* ids, const uint16_t* table, int64_t vocab, const uint16_t* visual,
                                int image_start, int nv, uint16_t* h, int T, int H, void* stream) {
  FFB_REQUIRE(ids && table && h, "ffb_embed_gather: NULL pointer");
  FFB_REQUIRE(T > 0 && H > 0 && H % 8 == 0, "ffb_embed_gather: bad shape T=%d H=%d", T, H);
  FFB_REQUIRE(!visual || (image_start >= 0 && nv >= 0 && image_start + nv <= T),
              "ffb_embed_gather: visual window [%d, %d) outside T=%d", image_start, image_start + nv, T);
  FFB_REQUIRE(ffb::aligned(table, 16) && ffb::aligned(h, 16) && (!visual || ffb::aligned(visual, 16)),
              "ffb_embed_gather: alignment");
  cudaError_t e = ffb::launch(embed_kernel, dim3(T), dim3(NT), 0, (cudaStream_t)stream, ids, table, vocab, visual,
                              image_start, nv, h, H);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_embed_gather: %s", cudaGetErrorString(e));
  return FFB_OK;
}

extern "C" int ffb_swiglu(const uint16_t* gate, const uint16_t* up, int row_stride, uint16_t* y, int M, int I,
                          void* stream) {
  FFB_REQUIRE(gate && up && y, "ffb_swiglu: NULL pointer");
  FFB_REQUIRE(M > 0 && I > 0 && row_stride >= I, "ffb_swiglu: bad shape");
  const size_t n = (size_t)M * I;
  int grid = (int)((n + NT - 1) / NT);
  if (grid > 148 * 16) grid = 148 * 16;
  cudaError_t e = ffb::launch(swiglu_kernel, dim3(grid), dim3(NT), 0, (cudaStream_t)stream, gate, up, row_stride, y,
                              M, I);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_swiglu: %s", cudaGetErrorString(e));
  return FFB_OK;
}

extern "C" int ffb_readout(const uint16_t* residual, const uint16_t* mlp, const float* mlp32, int splits,
                           const uint16_t* norm_w, float eps, const uint16_t* head, int n, int k, float* logits,
                           float* logprobs, int H, void* stream) {
  FFB_REQUIRE(residual && norm_w && head && logits, "ffb_readout: NULL pointer");
  FFB_REQUIRE(n >= 1 && n <= 8 && k >= 1 && k <= n, "ffb_readout: need 1 <= k <= n <= 8 (n=%d k=%d)", n, k);
  FFB_REQUIRE(H > 0 && H <= 12288, "ffb_readout: H=%d (max 12288)", H);
  FFB_REQUIRE(mlp || !mlp32 || splits >= 1, "ffb_readout: mlp32 needs splits >= 1");
  cudaError_t e = ffb::launch(readout_kernel, dim3(1), dim3(NT), (size_t)H * sizeof(float), (cudaStream_t)stream,
                              residual, mlp, mlp ? nullptr : mlp32, splits, norm_w, eps, head, n, k, logits, logprobs,
                              H);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_readout: %s", cudaGetErrorString(e));
  return FFB_OK;
}

namespace {
__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, const int64_t* __restrict__ index,
                                   uint8_t* __restrict__ dst, int row_bytes) {
  pdl_wait();
  pdl_launch();
  const int64_t r = index[blockIdx.x];
  const uint8_t* a = src + (size_t)r * row_bytes;
  uint8_t* b = dst + (size_t)blockIdx.x * row_bytes;
  for (int i = threadIdx.x; i < row_bytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(b)[i] = reinterpret_cast<const uint4*>(a)[i];
}
}  // namespace

extern "C" int ffb_gather_rows(const void* src, const int64_t* index, void* dst, int n, int row_bytes,
                               void* stream) {
  FFB_REQUIRE(src && index && dst, "ffb_gather_rows: NULL pointer");
  FFB_REQUIRE(n > 0 && row_bytes > 0 && row_bytes % 16 == 0, "ffb_gather_rows: row_bytes %d must be a multiple of 16",
              row_bytes);
  FFB_REQUIRE(ffb::aligned(src, 16) && ffb::aligned(dst, 16), "ffb_gather_rows: alignment");
  cudaError_t e = ffb::launch(gather_rows_kernel, dim3(n), dim3(128), 0, (cudaStream_t)stream, (const uint8_t*)src,
                              index, (uint8_t*)dst, row_bytes);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_gather_rows: %s", cudaGetErrorString(e));
  return FFB_OK;
}
