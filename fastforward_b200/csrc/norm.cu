// RMSNorm and residual-add + RMSNorm, each optionally emitting the FP8 copy of its
// output that the next linear consumes (so the quantiser needs no launch of its own).
//
// Rounding follows the reference kernels: x = bf16(a + b) (and bf16(x + deep) on the
// deepstack rows), y = bf16(bf16(x * inv) * w) (_legacy/lower_kernels.py:7-21,
// _legacy/sub10_runtime.py:31-36), with inv = 1/sqrt(sum(x^2)/H + eps) computed from an
// exact float64 sum of squares and IEEE sqrt/divide (order-independent, so the result is
// reproducible bit for bit; the reference's fp32 tree sum + hardware rsqrt is not).  One
// CTA per row with H/16 threads (two 128-bit vectors each: enough warps in flight to hide
// the memory latency), the row held in registers between the reduction and the stores.
// HBM traffic per row: read a, b (or the split-K partials), w; write residual, out, q8.
#include "common.cuh"
#include "pdl.cuh"
#include "peer.cuh"

namespace {

constexpr int MAXT = 512;   // threads per row: H/16 rounded up to a warp (two 8-element vectors each)
constexpr int MAXV = 2;     // 8-element vectors per thread -> H <= 8192

// Block-wide sum (float64) and max (float) over blockDim.x threads; every thread gets it.
__device__ __forceinline__ double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum_d(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double r = 0.0;
  for (int i = 0; i < nw; ++i) r += red[i];  // fixed order: identical in every thread
  __syncthreads();
  return r;
}

__device__ __forceinline__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_max(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = 0.f;
  for (int i = 0; i < nw; ++i) r = fmaxf(r, red[i]);
  __syncthreads();
  return r;
}

__device__ __forceinline__ void load8(const uint16_t* p, float (&f)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ void store8(uint16_t* p, const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = (uint32_t)f2bf(f[2 * i]) | ((uint32_t)f2bf(f[2 * i + 1]) << 16);
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}

struct NormArgs {
  const uint16_t* a;
  const uint16_t* b;
  const float* b32;
  int splits;
  const uint16_t* deep;
  int start, nv;
  const uint16_t* w;
  float eps;
  uint16_t* residual;
  uint16_t* out;
  int quant_mode;
  float inv_scale;
  uint8_t* q8;
  float* qscale;
  int T, H;
  int add;  // 0: plain RMSNorm of a
  // tensor-parallel ranks' partial planes (S == -2): planes[r] summed in rank order after
  // the row's handshake
  const float* planes[FFB_MAX_PEERS];
  ffb_peer_sync ps;
};

// S >= 1: b is the sum of S fp32 split-K partial planes (all loads issued before the first
// add, summed in plane order); S == 0: b is bf16 (or there is no add); S == -1: any number
// of planes, loaded plane by plane; S == -2: the tensor-parallel ranks' planes (peer
// memory), summed in rank order once the row's CTA has handshaken with every rank.
template <int V, int S>
__global__ void __launch_bounds__(MAXT) add_rmsnorm_kernel(const NormArgs p) {
  __shared__ float red[MAXT / 32];
  __shared__ double redd[MAXT / 32];
  const int NT = blockDim.x;
  const int nvec = p.H / 8;
  // the norm weight does not depend on the previous kernel: fetch it before waiting
  float w[V][8];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int v = threadIdx.x + i * NT;
    if (v < nvec) load8(p.w + v * 8, w[i]);
  }
  pdl_wait();
  pdl_launch();
  if constexpr (S == -2) {  // one handshake per CTA (slot = CTA), then its rows
    __shared__ int hs_ok;
    if (threadIdx.x == 0) {
      hs_ok = peer_handshake(p.ps, blockIdx.x);
      if (!hs_ok) atomicOr(&ffb_device_error_word, ffb::ERR_PEER_TIMEOUT);
    }
    __syncthreads();
    if (!hs_ok) return;
  }
  // one row per CTA (the peer variant's smaller grid strides over the rows)
  for (int row = blockIdx.x; row < p.T; row += gridDim.x) {
    const size_t base = (size_t)row * p.H;
    const bool deep_row = p.deep && row >= p.start && row < p.start + p.nv;
    float x[V][8], b[V][8];
    constexpr int SP = S > 0 ? S : 1;
    float4 part[V][SP][2];
    // every load of the row in flight before the first use
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int v = threadIdx.x + i * NT;
      if (v < nvec) {
        load8(p.a + base + v * 8, x[i]);
        if (p.add) {
          if constexpr (S == 0) {
            load8(p.b + base + v * 8, b[i]);
          } else if constexpr (S > 0) {
#pragma unroll
            for (int s = 0; s < S; ++s) {
              const float4* src = reinterpret_cast<const float4*>(p.b32 + (size_t)s * p.T * p.H + base + v * 8);
              part[i][s][0] = src[0];
              part[i][s][1] = src[1];
            }
          }
        }
      }
    }
    double ss = 0.0;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int v = threadIdx.x + i * NT;
      if (v < nvec) {
        if (p.add) {
          if constexpr (S != 0) {
#pragma unroll
            for (int e = 0; e < 8; ++e) b[i][e] = 0.f;
            auto add_plane = [&](const float4 lo, const float4 hi) {
              b[i][0] += lo.x; b[i][1] += lo.y; b[i][2] += lo.z; b[i][3] += lo.w;
              b[i][4] += hi.x; b[i][5] += hi.y; b[i][6] += hi.z; b[i][7] += hi.w;
            };
            if constexpr (S > 0) {
#pragma unroll
              for (int s = 0; s < S; ++s) add_plane(part[i][s][0], part[i][s][1]);
            } else if constexpr (S == -2) {
              for (int r = 0; r < p.ps.world; ++r) {
                const float4* src = reinterpret_cast<const float4*>(p.planes[r] + base + v * 8);
                add_plane(__ldcg(src), __ldcg(src + 1));
              }
            } else {
              for (int s = 0; s < p.splits; ++s) {
                const float4* src = reinterpret_cast<const float4*>(p.b32 + (size_t)s * p.T * p.H + base + v * 8);
                add_plane(src[0], src[1]);
              }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) b[i][e] = round_bf(b[i][e]);  // the linear's bf16 output
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) x[i][e] = round_bf(x[i][e] + b[i][e]);
          if (deep_row) {
            float d[8];
            load8(p.deep + (size_t)(row - p.start) * p.H + v * 8, d);
#pragma unroll
            for (int e = 0; e < 8; ++e) x[i][e] = round_bf(x[i][e] + d[e]);
          }
          if (p.residual) store8(p.residual + base + v * 8, x[i]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += (double)(x[i][e] * x[i][e]);  // x*x exact in fp32
      }
    }
    const float inv = inv_rms_from_ss(block_sum_d(ss, redd), p.H, p.eps);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int v = threadIdx.x + i * NT;
      if (v < nvec) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          x[i][e] = round_bf(round_bf(x[i][e] * inv) * w[i][e]);
          amax = fmaxf(amax, fabsf(x[i][e]));
        }
        if (p.out) store8(p.out + base + v * 8, x[i]);
      }
    }
    if (p.quant_mode == FFB_QUANT_NONE) continue;
    float mul = p.inv_scale, scale = 0.f, rcp = 0.f;
    if (p.quant_mode == FFB_QUANT_ROWWISE) {
      amax = block_max(amax, red);
      scale = fmaxf(amax, 1e-12f) / 448.f;
      rcp = __frcp_rn(scale);
      if (threadIdx.x == 0) p.qscale[row] = scale;
    }
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int v = threadIdx.x + i * NT;
      if (v < nvec) {
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const uint32_t b = p.quant_mode == FFB_QUANT_ROWWISE ? e4m3_quotient(x[i][e], scale, rcp)
                                                               : f2e4m3(clamp448(x[i][e] * mul));
          if (e < 4) lo |= b << (8 * e);
          else hi |= b << (8 * (e - 4));
        }
        *reinterpret_cast<uint2*>(p.q8 + base + v * 8) = make_uint2(lo, hi);
      }
    }
  }
}

int run(const NormArgs& p, const char* who, void* stream) {
  FFB_REQUIRE(p.a && p.w, "%s: NULL input", who);
  FFB_REQUIRE(p.T > 0 && p.H > 0 && p.H % 8 == 0 && p.H <= MAXT * MAXV * 8,
              "%s: H=%d must be a multiple of 8 and <= %d", who, p.H, MAXT * MAXV * 8);
  FFB_REQUIRE(p.quant_mode >= 0 && p.quant_mode <= 2, "%s: bad quant_mode %d", who, p.quant_mode);
  FFB_REQUIRE(p.quant_mode == FFB_QUANT_NONE || p.q8, "%s: quant_mode needs q8", who);
  FFB_REQUIRE(p.quant_mode != FFB_QUANT_ROWWISE || p.qscale, "%s: ROWWISE needs qscale", who);
  FFB_REQUIRE(p.out || p.quant_mode != FFB_QUANT_NONE, "%s: nothing to write", who);
  FFB_REQUIRE(ffb::aligned(p.a, 16) && ffb::aligned(p.w, 16) && (!p.out || ffb::aligned(p.out, 16)),
              "%s: bf16 rows must be 16-byte aligned", who);
  FFB_REQUIRE(!p.q8 || ffb::aligned(p.q8, 8), "%s: q8 must be 8-byte aligned", who);
  const int nvec = p.H / 8;
  int nt = (nvec + 1) / 2;     // two vectors per thread
  nt = (nt + 31) / 32 * 32;    // whole warps
  const bool planes = p.add && !p.b;
  const int sp = planes ? p.splits : 0;
  auto kernel = add_rmsnorm_kernel<MAXV, -1>;
  switch (p.ps.world > 0 ? -2 : sp) {
    case -2: kernel = add_rmsnorm_kernel<MAXV, -2>; break;
    case 0: kernel = add_rmsnorm_kernel<MAXV, 0>; break;
    case 1: kernel = add_rmsnorm_kernel<MAXV, 1>; break;
    case 2: kernel = add_rmsnorm_kernel<MAXV, 2>; break;
    case 3: kernel = add_rmsnorm_kernel<MAXV, 3>; break;
    case 4: kernel = add_rmsnorm_kernel<MAXV, 4>; break;
    default: break;
  }
  // the peer variant handshakes once per CTA: a grid of at most four CTAs per SM strides
  // over the rows
  const int sms4 = 4 * ffb::sm_count();
  const int grid = p.ps.world > 0 && p.T > sms4 ? sms4 : p.T;
  cudaError_t e = ffb::launch(kernel, dim3(grid), dim3(nt), 0, (cudaStream_t)stream, p);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "%s: launch: %s", who, cudaGetErrorString(e));
  return FFB_OK;
}

}  // namespace

extern "C" int ffb_rmsnorm(const uint16_t* x, const uint16_t* w, float eps, uint16_t* out, int quant_mode,
                           float inv_scale, uint8_t* q8, float* qscale, int T, int H, void* stream) {
  NormArgs p = {};
  p.a = x;
  p.w = w;
  p.eps = eps;
  p.out = out;
  p.quant_mode = quant_mode;
  p.inv_scale = inv_scale;
  p.q8 = q8;
  p.qscale = qscale;
  p.T = T;
  p.H = H;
  p.add = 0;
  return run(p, "ffb_rmsnorm", stream);
}

extern "C" int ffb_add_rmsnorm(const uint16_t* a, const uint16_t* b, const float* b32, int splits,
                               const uint16_t* deep, int start, int nv, const uint16_t* w, float eps,
                               uint16_t* residual, uint16_t* out, int quant_mode, float inv_scale, uint8_t* q8,
                               float* qscale, int T, int H, void* stream) {
  FFB_REQUIRE(b || (b32 && splits >= 1), "ffb_add_rmsnorm: need b or (b32, splits >= 1)");
  FFB_REQUIRE(!b32 || ffb::aligned(b32, 16), "ffb_add_rmsnorm: b32 must be 16-byte aligned");
  FFB_REQUIRE(!b || ffb::aligned(b, 16), "ffb_add_rmsnorm: b must be 16-byte aligned");
  FFB_REQUIRE(!deep || (start >= 0 && nv >= 0 && start + nv <= T && ffb::aligned(deep, 16)),
              "ffb_add_rmsnorm: bad deepstack window start=%d nv=%d T=%d", start, nv, T);
  FFB_REQUIRE(residual != nullptr, "ffb_add_rmsnorm: residual is NULL");
  NormArgs p = {};
  p.a = a;
  p.b = b;
  p.b32 = b ? nullptr : b32;
  p.splits = splits;
  p.deep = deep;
  p.start = start;
  p.nv = deep ? nv : 0;
  p.w = w;
  p.eps = eps;
  p.residual = residual;
  p.out = out;
  p.quant_mode = quant_mode;
  p.inv_scale = inv_scale;
  p.q8 = q8;
  p.qscale = qscale;
  p.T = T;
  p.H = H;
  p.add = 1;
  return run(p, "ffb_add_rmsnorm", stream);
}

extern "C" int ffb_add_rmsnorm_peers(const uint16_t* a, const float* const* planes, const ffb_peer_sync* sync,
                                     const uint16_t* deep, int start, int nv, const uint16_t* w, float eps,
                                     uint16_t* residual, uint16_t* out, int quant_mode, float inv_scale, uint8_t* q8,
                                     float* qscale, int T, int H, void* stream) {
  FFB_REQUIRE(planes && sync, "ffb_add_rmsnorm_peers: NULL planes / sync");
  FFB_REQUIRE(sync->world >= 1 && sync->world <= FFB_MAX_PEERS && sync->rank >= 0 && sync->rank < sync->world,
              "ffb_add_rmsnorm_peers: rank %d of %d (at most %d ranks)", sync->rank, sync->world, FFB_MAX_PEERS);
  FFB_REQUIRE(sync->local && T <= sync->nslots, "ffb_add_rmsnorm_peers: %d rows need %d slots (have %d)", T, T,
              sync->nslots);
  for (int r = 0; r < sync->world; ++r)
    FFB_REQUIRE(planes[r] && sync->flags[r] && ffb::aligned(planes[r], 16),
                "ffb_add_rmsnorm_peers: rank %d's plane / flags missing or unaligned", r);
  FFB_REQUIRE(!deep || (start >= 0 && nv >= 0 && start + nv <= T && ffb::aligned(deep, 16)),
              "ffb_add_rmsnorm_peers: bad deepstack window start=%d nv=%d T=%d", start, nv, T);
  FFB_REQUIRE(residual != nullptr, "ffb_add_rmsnorm_peers: residual is NULL");
  NormArgs p = {};
  p.a = a;
  p.splits = 1;
  p.deep = deep;
  p.start = start;
  p.nv = deep ? nv : 0;
  p.w = w;
  p.eps = eps;
  p.residual = residual;
  p.out = out;
  p.quant_mode = quant_mode;
  p.inv_scale = inv_scale;
  p.q8 = q8;
  p.qscale = qscale;
  p.T = T;
  p.H = H;
  p.add = 1;
  for (int r = 0; r < sync->world; ++r) p.planes[r] = planes[r];
  p.ps = *sync;
  return run(p, "ffb_add_rmsnorm_peers", stream);
}
