// FP8 quantisers: activations (static per-tensor scale or per-token dynamic scale),
// set-up-time weights (per-tensor or per-output-channel absmax), and the gate/up row
// interleave used by the fused SwiGLU GEMM epilogue.
//
// Static:   q = e4m3(clamp(x * inv, +-448))              _family/depth_fp8.py:8-12
// Rowwise:  s = max(max|x|, 1e-12)/448, q = e4m3(x / s)    _legacy/fp8_private.py:11-18
// Weights:  s = max(max|W|, 1e-12)/448, W8 = e4m3(W / s)   _legacy/limit_kernels.py:122-127
//                                       (per row: _legacy/fp8_private.py:22-27)
// All divisions are IEEE round-to-nearest (__fdiv_rn), all conversions RNE, so the bytes
// are reproducible on any IEEE implementation.
#include "common.cuh"
#include "pdl.cuh"
#include "peer.cuh"

#include <atomic>

namespace {

constexpr int NT = 256;

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float r = lane < NT / 32 ? red[lane] : 0.f;
    r = warp_max(r);
    if (lane == 0) red[NT / 32] = r;
  }
  __syncthreads();
  const float r = red[NT / 32];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float block_max_any(float v, float* red) {  // blockDim.x threads
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < nw; ++i) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}

// One CTA per row, the row held in registers as 8-element vectors (QV per thread):
// absmax (ROWWISE only), then quantise with 8-byte stores.  K % 8 == 0.
constexpr int QV = 2;
__global__ void __launch_bounds__(1024) quant_rows_vec_kernel(const uint16_t* __restrict__ x, int mode, float inv,
                                                             uint8_t* __restrict__ q8, float* __restrict__ qscale,
                                                             int K) {
  __shared__ float red[32];
  pdl_wait();
  pdl_launch();
  const int row = blockIdx.x, nvec = K / 8;
  const uint16_t* xr = x + (size_t)row * K;
  uint8_t* qr = q8 + (size_t)row * K;
  float v[QV][8];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < QV; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      const uint4 u = *reinterpret_cast<const uint4*>(xr + vi * 8);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[i][2 * e] = __uint_as_float(w[e] << 16);
        v[i][2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[i][e]));
    }
  }
  float scale = 0.f;
  if (mode == FFB_QUANT_ROWWISE) {
    amax = block_max_any(amax, red);
    scale = fmaxf(amax, 1e-12f) / 448.f;
    if (threadIdx.x == 0) qscale[row] = scale;
  } else if (mode == FFB_QUANT_ROWSCALE) {
    scale = qscale[row];
  }
  const float rcp = __frcp_rn(scale);
#pragma unroll
  for (int i = 0; i < QV; ++i) {
    const int vi = threadIdx.x + i * blockDim.x;
    if (vi < nvec) {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        // ROWSCALE's given scale is outside e4m3_quotient's checked domain: IEEE divide
        const uint32_t b = mode == FFB_QUANT_ROWWISE   ? e4m3_quotient(v[i][e], scale, rcp)
                           : mode == FFB_QUANT_STATIC ? f2e4m3(clamp448(v[i][e] * inv))
                                                      : f2e4m3(clamp448(__fdiv_rn(v[i][e], scale)));
        if (e < 4) lo |= b << (8 * e);
        else hi |= b << (8 * (e - 4));
      }
      *reinterpret_cast<uint2*>(qr + vi * 8) = make_uint2(lo, hi);
    }
  }
}

// Rowwise quantiser of rows split over the tensor-parallel ranks.  A grid of at most four
// CTAs per SM strides over the rows twice: first each row's slice maximum goes to every
// rank's amax[p][rank][row] (peer stores); then the CTA handshakes its slot with every rank
// (one handshake per CTA), and each row is quantised with max(max over the ranks' maxima,
// 1e-12) / 448 as its scale.
struct PeerAmax {
  float* amax[FFB_MAX_PEERS];  // rank p's [world][M] buffer, as mapped here
};
__device__ __forceinline__ void load_row8(const uint16_t* xr, int vi, float (&v)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(xr + vi * 8);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    v[2 * e] = __uint_as_float(w[e] << 16);
    v[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
  }
}
__global__ void __launch_bounds__(1024) quant_rows_peer_kernel(const uint16_t* __restrict__ x, PeerAmax pa,
                                                              ffb_peer_sync ps, uint8_t* __restrict__ q8,
                                                              float* __restrict__ qscale, int M, int K) {
  __shared__ float red[32];
  __shared__ int hs_ok;
  pdl_wait();
  pdl_launch();
  const int nvec = K / 8;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const uint16_t* xr = x + (size_t)row * K;
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < QV; ++i) {
      const int vi = threadIdx.x + i * blockDim.x;
      if (vi < nvec) {
        float v[8];
        load_row8(xr, vi, v);
#pragma unroll
        for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[e]));
      }
    }
    amax = block_max_any(amax, red);
    if (threadIdx.x < ps.world) {
      pa.amax[threadIdx.x][(size_t)ps.rank * M + row] = amax;
      fence_acq_rel_sys();
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    hs_ok = peer_handshake(ps, blockIdx.x);  // fences the maxima above before its signals
    if (!hs_ok) atomicOr(&ffb_device_error_word, ffb::ERR_PEER_TIMEOUT);
  }
  __syncthreads();
  if (!hs_ok) return;
  for (int row = blockIdx.x; row < M; row += gridDim.x) {
    const uint16_t* xr = x + (size_t)row * K;
    uint8_t* qr = q8 + (size_t)row * K;
    float m = 0.f;
    for (int q = 0; q < ps.world; ++q) m = fmaxf(m, __ldcg(pa.amax[ps.rank] + (size_t)q * M + row));
    const float scale = fmaxf(m, 1e-12f) / 448.f, rcp = __frcp_rn(scale);
    if (threadIdx.x == 0) qscale[row] = scale;
#pragma unroll
    for (int i = 0; i < QV; ++i) {
      const int vi = threadIdx.x + i * blockDim.x;
      if (vi < nvec) {
        float v[8];
        load_row8(xr, vi, v);
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint32_t b = e4m3_quotient(v[e], scale, rcp);
          if (e < 4) lo |= b << (8 * e);
          else hi |= b << (8 * (e - 4));
        }
        *reinterpret_cast<uint2*>(qr + vi * 8) = make_uint2(lo, hi);
      }
    }
  }
}

// Scalar fallback for any K: absmax pass, then quantise.
__global__ void __launch_bounds__(NT) quant_rows_kernel(const uint16_t* __restrict__ x, int mode, float inv,
                                                        uint8_t* __restrict__ q8, float* __restrict__ qscale,
                                                        int K) {
  __shared__ float red[NT / 32 + 1];
  pdl_wait();
  pdl_launch();
  const int row = blockIdx.x;
  const uint16_t* xr = x + (size_t)row * K;
  uint8_t* qr = q8 + (size_t)row * K;
  float scale = 0.f;
  if (mode == FFB_QUANT_ROWWISE) {
    float amax = 0.f;
    for (int k = threadIdx.x; k < K; k += NT) amax = fmaxf(amax, fabsf(bf2f(xr[k])));
    amax = block_max(amax, red);
    scale = fmaxf(amax, 1e-12f) / 448.f;
    if (threadIdx.x == 0) qscale[row] = scale;
  } else if (mode == FFB_QUANT_ROWSCALE) {
    scale = qscale[row];
  }
  const float rcp = __frcp_rn(scale);
  for (int k = threadIdx.x; k < K; k += NT) {
    const float v = bf2f(xr[k]);
    qr[k] = mode == FFB_QUANT_ROWWISE   ? e4m3_quotient(v, scale, rcp)
            : mode == FFB_QUANT_STATIC ? f2e4m3(clamp448(v * inv))
                                       : f2e4m3(clamp448(__fdiv_rn(v, scale)));
  }
}

// Weight absmax per row into ws (fp32), or the global max when `reduce_rows` > 0.
__global__ void __launch_bounds__(NT) row_absmax_kernel(const uint16_t* __restrict__ w, float* __restrict__ out,
                                                        int K) {
  __shared__ float red[NT / 32 + 1];
  pdl_wait();
  pdl_launch();
  const uint16_t* wr = w + (size_t)blockIdx.x * K;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += NT) amax = fmaxf(amax, fabsf(bf2f(wr[k])));
  amax = block_max(amax, red);
  if (threadIdx.x == 0) out[blockIdx.x] = amax;
}

__global__ void __launch_bounds__(NT) global_scale_kernel(const float* __restrict__ rowmax, int N,
                                                          float* __restrict__ scale) {
  __shared__ float red[NT / 32 + 1];
  pdl_wait();
  pdl_launch();
  float m = 0.f;
  for (int i = threadIdx.x; i < N; i += NT) m = fmaxf(m, rowmax[i]);
  m = block_max(m, red);
  if (threadIdx.x == 0) scale[0] = fmaxf(m, 1e-12f) / 448.f;
}

// W8[n,k] = e4m3(clamp(W / s)), s = scale[per_channel ? n : 0]; per-channel scales are
// produced here from rowmax.
__global__ void __launch_bounds__(NT) weight_quant_kernel(const uint16_t* __restrict__ w,
                                                          const float* __restrict__ rowmax, int per_channel,
                                                          float* __restrict__ scale, uint8_t* __restrict__ w8,
                                                          int K) {
  pdl_wait();
  pdl_launch();
  const int n = blockIdx.x;
  float s;
  if (per_channel) {
    s = fmaxf(rowmax[n], 1e-12f) / 448.f;
    if (threadIdx.x == 0) scale[n] = s;
  } else {
    s = scale[0];
  }
  const uint16_t* wr = w + (size_t)n * K;
  uint8_t* qr = w8 + (size_t)n * K;
  for (int k = threadIdx.x; k < K; k += NT) qr[k] = f2e4m3(clamp448(__fdiv_rn(bf2f(wr[k]), s)));
}

// Row permutation for the SwiGLU epilogue: dst tile t = src gate rows [128t, 128t+128)
// then src up rows [I + 128t, I + 128t + 128).  One CTA per destination row.
__global__ void pack_gateup_kernel(const uint8_t* __restrict__ src, uint8_t* __restrict__ dst, int I,
                                   size_t row_bytes) {
  pdl_wait();
  pdl_launch();
  const int r = blockIdx.x;
  const int t = r / 256, j = r % 256;
  const int s = j < 128 ? 128 * t + j : I + 128 * t + (j - 128);
  const uint8_t* a = src + (size_t)s * row_bytes;
  uint8_t* b = dst + (size_t)r * row_bytes;
  if (row_bytes % 16 == 0) {
    for (size_t i = threadIdx.x; i < row_bytes / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(b)[i] = reinterpret_cast<const uint4*>(a)[i];
  } else {
    for (size_t i = threadIdx.x; i < row_bytes; i += blockDim.x) b[i] = a[i];
  }
}

}  // namespace

extern "C" int ffb_quantize_fp8(const uint16_t* x, int quant_mode, float inv_scale, uint8_t* q8, float* qscale,
                                int M, int K, void* stream) {
  FFB_REQUIRE(x && q8, "ffb_quantize_fp8: NULL pointer");
  FFB_REQUIRE(M > 0 && K > 0, "ffb_quantize_fp8: bad shape M=%d K=%d", M, K);
  FFB_REQUIRE(quant_mode == FFB_QUANT_STATIC || quant_mode == FFB_QUANT_ROWWISE || quant_mode == FFB_QUANT_ROWSCALE,
              "ffb_quantize_fp8: bad mode %d", quant_mode);
  FFB_REQUIRE(quant_mode == FFB_QUANT_STATIC || qscale, "ffb_quantize_fp8: ROWWISE / ROWSCALE need qscale");
  cudaError_t e;
  const int nvec = K / 8;
  if (K % 8 == 0 && ffb::aligned(x, 16) && ffb::aligned(q8, 8) && nvec <= 1024 * QV) {
    int nt = (nvec + QV - 1) / QV;
    nt = (nt + 31) / 32 * 32;
    e = ffb::launch(quant_rows_vec_kernel, dim3(M), dim3(nt), 0, (cudaStream_t)stream, x, quant_mode, inv_scale, q8,
                    qscale, K);
  } else {
    e = ffb::launch(quant_rows_kernel, dim3(M), dim3(NT), 0, (cudaStream_t)stream, x, quant_mode, inv_scale, q8,
                    qscale, K);
  }
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_quantize_fp8: %s", cudaGetErrorString(e));
  return FFB_OK;
}

extern "C" int ffb_quantize_weight_fp8(const uint16_t* w, int per_channel, uint8_t* w8, float* scale, void* ws,
                                       int N, int K, void* stream) {
  FFB_REQUIRE(w && w8 && scale && ws, "ffb_quantize_weight_fp8: NULL pointer");
  FFB_REQUIRE(N > 0 && K > 0, "ffb_quantize_weight_fp8: bad shape N=%d K=%d", N, K);
  cudaStream_t s = (cudaStream_t)stream;
  float* rowmax = reinterpret_cast<float*>(ws);
  cudaError_t e = ffb::launch(row_absmax_kernel, dim3(N), dim3(NT), 0, s, w, rowmax, K);
  if (e == cudaSuccess && !per_channel)
    e = ffb::launch(global_scale_kernel, dim3(1), dim3(NT), 0, s, (const float*)rowmax, N, scale);
  if (e == cudaSuccess)
    e = ffb::launch(weight_quant_kernel, dim3(N), dim3(NT), 0, s, w, (const float*)rowmax, per_channel, scale, w8, K);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_quantize_weight_fp8: %s", cudaGetErrorString(e));
  return FFB_OK;
}

// Fixed scratch of ffb_quantize_weight_fp8_noalloc: the weight's per-row |max|, one fp32
// per row.  No entry needs a starting value: row_absmax_kernel writes rows [0, N) before
// global_scale_kernel / weight_quant_kernel read them, in stream order.
static __device__ __align__(256) float g_noalloc_rowmax[FFB_QW_NOALLOC_MAX_N];

namespace {
constexpr int kMaxDevices = 64;
std::atomic<float*> g_noalloc_rowmax_ptr[kMaxDevices];  // per device, looked up once
}  // namespace

extern "C" int ffb_quantize_weight_fp8_noalloc(const uint16_t* w, int per_channel, uint8_t* w8, float* scale,
                                               int N, int K, void* stream) {
  FFB_REQUIRE(w && w8 && scale, "ffb_quantize_weight_fp8_noalloc: NULL pointer");
  FFB_REQUIRE(N > 0 && K > 0, "ffb_quantize_weight_fp8_noalloc: bad shape N=%d K=%d", N, K);
  FFB_REQUIRE(N <= FFB_QW_NOALLOC_MAX_N,
              "ffb_quantize_weight_fp8_noalloc: N=%d rows exceed the fixed scratch of %d rows "
              "(use ffb_quantize_weight_fp8 with caller scratch)", N, FFB_QW_NOALLOC_MAX_N);
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_quantize_weight_fp8_noalloc: cudaGetDevice: %s",
                                         cudaGetErrorString(e));
  FFB_REQUIRE(dev >= 0 && dev < kMaxDevices, "ffb_quantize_weight_fp8_noalloc: device %d out of range", dev);
  float* rowmax = g_noalloc_rowmax_ptr[dev].load(std::memory_order_acquire);
  if (rowmax == nullptr) {
    // with `dev` current; concurrent first calls all store the same address
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&rowmax), g_noalloc_rowmax);
    if (e != cudaSuccess)
      return ffb::fail(FFB_ECUDA, "ffb_quantize_weight_fp8_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_noalloc_rowmax_ptr[dev].store(rowmax, std::memory_order_release);
  }
  cudaStream_t s = (cudaStream_t)stream;
  e = ffb::launch(row_absmax_kernel, dim3(N), dim3(NT), 0, s, w, rowmax, K);
  if (e == cudaSuccess && !per_channel)
    e = ffb::launch(global_scale_kernel, dim3(1), dim3(NT), 0, s, (const float*)rowmax, N, scale);
  if (e == cudaSuccess)
    e = ffb::launch(weight_quant_kernel, dim3(N), dim3(NT), 0, s, w, (const float*)rowmax, per_channel, scale, w8, K);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_quantize_weight_fp8_noalloc: %s", cudaGetErrorString(e));
  return FFB_OK;
}

extern "C" int ffb_pack_gateup(const void* src, void* dst, int I, int K, int elem_bytes, void* stream) {
  FFB_REQUIRE(src && dst && src != dst, "ffb_pack_gateup: bad pointers");
  FFB_REQUIRE(I > 0 && I % 128 == 0, "ffb_pack_gateup: I=%d must be a multiple of 128", I);
  FFB_REQUIRE(elem_bytes == 1 || elem_bytes == 2 || elem_bytes == 4, "ffb_pack_gateup: elem_bytes %d", elem_bytes);
  FFB_REQUIRE(K > 0, "ffb_pack_gateup: K=%d", K);
  const size_t row_bytes = (size_t)K * elem_bytes;
  FFB_REQUIRE(row_bytes % 16 != 0 || (ffb::aligned(src, 16) && ffb::aligned(dst, 16)),
              "ffb_pack_gateup: rows must be 16-byte aligned");
  cudaError_t e = ffb::launch(pack_gateup_kernel, dim3(2 * I), dim3(128), 0, (cudaStream_t)stream,
                              (const uint8_t*)src, (uint8_t*)dst, I, row_bytes);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_pack_gateup: %s", cudaGetErrorString(e));
  return FFB_OK;
}

extern "C" int ffb_quantize_fp8_peers(const uint16_t* x, float* const* amax, const ffb_peer_sync* sync, uint8_t* q8,
                                      float* qscale, int M, int K, void* stream) {
  FFB_REQUIRE(x && amax && sync && q8 && qscale, "ffb_quantize_fp8_peers: NULL pointer");
  FFB_REQUIRE(M > 0 && K > 0 && K % 8 == 0 && K / 8 <= 1024 * QV, "ffb_quantize_fp8_peers: bad shape M=%d K=%d", M, K);
  FFB_REQUIRE(ffb::aligned(x, 16) && ffb::aligned(q8, 8), "ffb_quantize_fp8_peers: alignment");
  FFB_REQUIRE(sync->world >= 1 && sync->world <= FFB_MAX_PEERS && sync->rank >= 0 && sync->rank < sync->world,
              "ffb_quantize_fp8_peers: rank %d of %d (at most %d ranks)", sync->rank, sync->world, FFB_MAX_PEERS);
  FFB_REQUIRE(sync->local && M <= sync->nslots, "ffb_quantize_fp8_peers: %d rows need %d slots (have %d)", M, M,
              sync->nslots);
  PeerAmax pa = {};
  for (int r = 0; r < sync->world; ++r) {
    FFB_REQUIRE(amax[r] && sync->flags[r], "ffb_quantize_fp8_peers: rank %d's amax / flags missing", r);
    pa.amax[r] = amax[r];
  }
  int nt = (K / 8 + QV - 1) / QV;
  nt = (nt + 31) / 32 * 32;
  const int grid = M < 4 * ffb::sm_count() ? M : 4 * ffb::sm_count();
  cudaError_t e = ffb::launch(quant_rows_peer_kernel, dim3(grid), dim3(nt), 0, (cudaStream_t)stream, x, pa, *sync,
                              q8, qscale, M, K);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_quantize_fp8_peers: %s", cudaGetErrorString(e));
  return FFB_OK;
}
