// FP8 e4m3 W8A8 linear on the sm_100a tensor cores (tcgen05, kind::f8f6f4).
//
// Replaces the reference's quantiser + torch._scaled_mm pair
// (_family/depth_fp8.py:22-26, _legacy/fp8_private.py:29-38) and, for the qkv projection,
// also the QK-norm + RoPE kernel that follows it (_legacy/broad_kernels.py:63-74).
//
// Tile = 128 tokens (UMMA M) x BN output features (UMMA N = 256, or 128 for one attention
// head).  A tcgen05.mma of kind::f8f6f4 costs a near-constant ~100 ns whatever its N up to
// 256, so the wide dimension goes on N; D[token, feature] accumulates in tensor memory
// (fp32, lane = token, column = feature) and every fused epilogue is thread-local: a
// thread owns one token's row of the tile.
//
// Persistent kernel, one CTA per SM, tiles assigned round-robin (token tile fastest, so
// the CTAs that share a weight tile run together and it streams from HBM once).
// Roles (320 threads):
//   warp 0      TMA producer: activation tile + weight tile per 128-byte K block into a
//               ring of STAGES shared-memory slots (full[s] / empty[s] mbarriers); the
//               weight half of the first ring pass is requested before the programmatic-
//               launch wait (weights do not depend on the previous kernel);
//   warp 1      TMEM allocator + single-thread MMA issuer; two accumulator buffers so the
//               MMAs of tile i+1 overlap the epilogue of tile i (tfull[b] / tempty[b]);
//   warps 2..17 epilogue:
//               warp w reads TMEM lanes 32*(w%4).. (its 32 tokens) and its share of
//               the columns, applies per-token x per-feature scales and writes:
//               bf16 rows / fp32 split-K partial rows / SwiGLU rows / (qkv) per-head
//               RMSNorm + rotate-half RoPE rows, head-major.
// Every wait is bounded (mbar_wait_bounded); a timeout sets the CTA abort flag and the
// device error word; all roles unwind, in-flight copies and MMAs drain, TMEM is released.
#include "common.cuh"
#include "pdl.cuh"

#include <string.h>

namespace {

constexpr int BM = 128;      // tokens per tile (UMMA M)
constexpr int BK = 128;      // K bytes per stage (one 128-byte swizzle atom row)
constexpr int UMMA_K = 32;   // K per tcgen05.mma for 8-bit operands
constexpr int A_TILE_BYTES = BM * BK;
constexpr int SMEM_LIMIT = 232448;
constexpr int EPI_QKROPE = 100;  // internal epilogue code of ffb_fp8_gemm_qk_rope
constexpr int EPI_SWIGLU_Q8 = 101;  // internal epilogue code of ffb_fp8_gemm_swiglu_fp8
// Epilogue warps per instance: four per TMEM lane quarter.
__host__ __device__ constexpr int epi_warps(int) { return 16; }
__host__ __device__ constexpr int threads_of(int epi) { return 64 + epi_warps(epi) * 32; }

template <int BN>
struct Cfg {
  static constexpr int B_TILE_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_TILE_BYTES + B_TILE_BYTES;
  static constexpr int STG_BYTES = 16 * 2048;  // 16 x [32 rows x 64 B] store staging buffers
  static constexpr int FIXED = STG_BYTES + 256 + 1024;    // staging, barriers, alignment slack
  static constexpr int FIT = (SMEM_LIMIT - FIXED) / STAGE_BYTES;
  static constexpr int STAGES = FIT > 8 ? 8 : FIT;
  static constexpr int SMEM = STAGES * STAGE_BYTES + FIXED;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulator buffers
  static_assert(BN == 128 || BN == 256, "feature tile must be 128 or 256");
};

struct RopeSide {
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  const uint16_t* cos;
  const uint16_t* sin;
  uint16_t* yq;
  uint16_t* yk;
  uint16_t* yv;
  float eps;
  int HQ, HK;
};

// The fused prologue (FFB_PRO_*): bf16 rows -> the GEMM's FP8 operand and row scales.
struct ProArgs {
  const uint16_t* x;    // QUANT: source rows; ADD_RMSNORM: residual input a
  const uint16_t* b;    // bf16 addend or NULL
  const float* b32;     // fp32 split partials [splits][M][K] when b is NULL
  int splits, add;
  const uint16_t* deep;
  int start, nv;
  const uint16_t* w;    // RMSNorm weight
  float eps;
  uint16_t* residual;
  int quant_mode;
  float inv;
  uint8_t* q8;          // = the GEMM's A operand
  float* qscale;        // ROWWISE: = the GEMM's per-row A scale
  uint64_t* sync;       // grid barrier word
};

struct GemmArgs {
  const float* a_scale;
  const float* w_scale;
  uint16_t* out;
  float* ws;
  int a_per_row, w_per_col, epilogue;
  int M, N, K, n_ttiles, splits, n_tiles;
  float out_inv;  // EPI_SWIGLU_Q8: static inverse scale of the next linear's input
  RopeSide rope;
  ProArgs pro;
};

constexpr int PRO_NONE = 0;
constexpr int PRO_ROWS = 4;        // rows per prologue batch (at most)
constexpr int PRO_ITEMS_Q = 8;     // 8-element vectors per thread and batch: QUANT
constexpr int PRO_ITEMS_N = 2;     //                                         ADD_RMSNORM
constexpr int PRO_MAX_SPLITS = 8;
__host__ __device__ constexpr int pro_items(int pro) { return pro == FFB_PRO_QUANT ? PRO_ITEMS_Q : PRO_ITEMS_N; }

// Slot-indexed register arrays: the row slot of an item is a run-time value, so select
// it with unrolled compares instead of dynamic indexing (which would go to local memory).
template <typename T, int N>
__device__ __forceinline__ void slot_add(T (&a)[N], int k, T v) {
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i == k) a[i] += v;
}
template <int N>
__device__ __forceinline__ void slot_max(float (&a)[N], int k, float v) {
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (i == k) a[i] = fmaxf(a[i], v);
}
template <typename T, int N>
__device__ __forceinline__ T slot_get(const T (&a)[N], int k) {
  T r = a[0];
#pragma unroll
  for (int i = 1; i < N; ++i)
    if (i == k) r = a[i];
  return r;
}
__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = (uint32_t)f2bf(f[2 * i]) | ((uint32_t)f2bf(f[2 * i + 1]) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// Per-row statistics of a prologue batch: every thread adds its items' contributions into
// PRO_ROWS register slots; the block reduces them (warp shuffles, then one thread per row
// over the warps' partials, fixed order) and that thread derives the row's values into
// shared memory, where every thread reads them by row index.
//   sum:  v = exact float64 sum of squares  -> out[r] = 1/rms (inv_rms_from_ss)
//   max:  v = max |y|                        -> out[r] = scale = max(v, 1e-12)/448
// red: NW * PRO_ROWS doubles; out: PRO_ROWS floats (shared memory).
__device__ __forceinline__ void row_inv_rms(const double (&v)[PRO_ROWS], int n, int K, float eps, double* red,
                                            float* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int r = 0; r < PRO_ROWS; ++r) {
    if (r < n) {
      const double t = warp_sum_d(v[r]);
      if (lane == 0) red[warp * PRO_ROWS + r] = t;
    }
  }
  __syncthreads();
  if ((int)threadIdx.x < n) {
    double t = 0.0;
    for (int w = 0; w < nw; ++w) t += red[w * PRO_ROWS + threadIdx.x];
    out[threadIdx.x] = inv_rms_from_ss(t, K, eps);
  }
  __syncthreads();
}
__device__ __forceinline__ void row_scales(const float (&v)[PRO_ROWS], int n, float* red, float* out) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
#pragma unroll
  for (int r = 0; r < PRO_ROWS; ++r) {
    if (r < n) {
      const float t = warp_max(v[r]);
      if (lane == 0) red[warp * PRO_ROWS + r] = t;
    }
  }
  __syncthreads();
  if ((int)threadIdx.x < n) {
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t = fmaxf(t, red[w * PRO_ROWS + threadIdx.x]);
    out[threadIdx.x] = fmaxf(t, 1e-12f) / 448.f;
  }
  __syncthreads();
}

// The fused prologue: CTA c owns rows [c*M/G, (c+1)*M/G) and processes them in batches of
// up to PRO_ROWS rows, the batch's 8-element vectors spread over all threads (at most
// pro_items(PRO) per thread).  Each batch first issues every load it needs (so their
// latencies overlap), then computes.  The arithmetic is that of add_rmsnorm_kernel
// (norm.cu) and quant_rows_vec_kernel (quant.cu), element for element, so the bytes are
// the same:
//   ADD_RMSNORM: x = bf16(a + bf16(sum of partials in split order) | b) (+ deep:
//                bf16(x + d)), inv = 1/sqrt(sum(x^2)/K + eps) (exact float64 sum),
//                y = bf16(bf16(x inv) w);
//   QUANT:       y = the bf16 input row;
//   then STATIC q = e4m3(clamp(y * inv_scale)), ROWWISE s = max(max|y|, 1e-12)/448,
//   q = e4m3(y / s) with an IEEE divide.
// `issue_prefetch()` is called once by every thread right after the first batch's loads
// are in flight (the caller's weight prefetch then queues behind them).
// scratch: NW * PRO_ROWS doubles + PRO_ROWS floats of shared memory.
template <int PRO, typename F>
__device__ void prologue_rows(const GemmArgs& g, uint8_t* scratch, F&& issue_prefetch) {
  constexpr int ITEMS = pro_items(PRO);
  const ProArgs& p = g.pro;
  const int M = g.M, K = g.K, nvec = K >> 3, NT = blockDim.x, G = gridDim.x, c = blockIdx.x;
  const int r_begin = (int)((long long)c * M / G), r_end = (int)((long long)(c + 1) * M / G);
  int rb_max = ITEMS * NT / nvec;
  rb_max = rb_max > PRO_ROWS ? PRO_ROWS : rb_max;  // >= 1 (host check)
  double* red_d = reinterpret_cast<double*>(scratch);
  float* red_f = reinterpret_cast<float*>(scratch);
  float* stat = reinterpret_cast<float*>(scratch + (NT >> 5) * PRO_ROWS * sizeof(double));
  const bool rowwise = p.quant_mode == FFB_QUANT_ROWWISE;
  bool prefetched = false;
  if (r_begin >= r_end) {
    issue_prefetch();
    prefetched = true;
  }
  for (int r0 = r_begin; r0 < r_end; r0 += rb_max) {
    const int rb = r_end - r0 < rb_max ? r_end - r0 : rb_max;
    const int items = rb * nvec;
    uint4 xv[ITEMS];  // the bf16 rows to quantise (after the norm, for ADD_RMSNORM)
    float amax[PRO_ROWS];
#pragma unroll
    for (int r = 0; r < PRO_ROWS; ++r) amax[r] = 0.f;
    if constexpr (PRO == FFB_PRO_ADD_RMSNORM) {
      // ---- loads: residual row, norm weight, bf16 addend
      uint4 wv[ITEMS];
      float bs[ITEMS][8];
#pragma unroll
      for (int j = 0; j < ITEMS; ++j) {
        const int i = threadIdx.x + j * NT;
#pragma unroll
        for (int e = 0; e < 8; ++e) bs[j][e] = 0.f;
        if (i < items) {
          const int rr = i / nvec, v = i - rr * nvec;
          const size_t off = (size_t)(r0 + rr) * K + (size_t)v * 8;
          xv[j] = *reinterpret_cast<const uint4*>(p.x + off);
          wv[j] = __ldg(reinterpret_cast<const uint4*>(p.w + (size_t)v * 8));
          if (p.add && p.b) unpack8(*reinterpret_cast<const uint4*>(p.b + off), bs[j]);
        }
      }
      if (!prefetched) {
        issue_prefetch();
        prefetched = true;
      }
      // ---- split-K partials, summed in split order; two splits of every item per round trip
      if (p.add && !p.b) {
#pragma unroll 1
        for (int s0 = 0; s0 < p.splits; s0 += 2) {
          float4 lo[ITEMS][2], hi[ITEMS][2];
#pragma unroll
          for (int j = 0; j < ITEMS; ++j) {
            const int i = threadIdx.x + j * NT;
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              if (i < items && s0 + u < p.splits) {
                const int rr = i / nvec, v = i - rr * nvec;
                const float4* src =
                    reinterpret_cast<const float4*>(p.b32 + ((size_t)(s0 + u) * M + r0 + rr) * K + (size_t)v * 8);
                lo[j][u] = __ldcg(src);
                hi[j][u] = __ldcg(src + 1);
              }
            }
          }
#pragma unroll
          for (int j = 0; j < ITEMS; ++j) {
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              if (s0 + u < p.splits) {
                bs[j][0] += lo[j][u].x; bs[j][1] += lo[j][u].y; bs[j][2] += lo[j][u].z; bs[j][3] += lo[j][u].w;
                bs[j][4] += hi[j][u].x; bs[j][5] += hi[j][u].y; bs[j][6] += hi[j][u].z; bs[j][7] += hi[j][u].w;
              }
            }
          }
        }
      }
      // ---- residual x, its sum of squares
      double ss[PRO_ROWS];
#pragma unroll
      for (int r = 0; r < PRO_ROWS; ++r) ss[r] = 0.0;
#pragma unroll
      for (int j = 0; j < ITEMS; ++j) {
        const int i = threadIdx.x + j * NT;
        if (i < items) {
          const int rr = i / nvec, v = i - rr * nvec, row = r0 + rr;
          float x[8];
          unpack8(xv[j], x);
          if (p.add) {
#pragma unroll
            for (int e = 0; e < 8; ++e) x[e] = round_bf(x[e] + round_bf(bs[j][e]));  // the linear's bf16 output
            if (p.deep && row >= p.start && row < p.start + p.nv) {  // deepstack rows (first layers only)
              float d[8];
              unpack8(*reinterpret_cast<const uint4*>(p.deep + (size_t)(row - p.start) * K + (size_t)v * 8), d);
#pragma unroll
              for (int e = 0; e < 8; ++e) x[e] = round_bf(x[e] + d[e]);
            }
            xv[j] = pack8(x);
            if (p.residual) *reinterpret_cast<uint4*>(p.residual + (size_t)row * K + (size_t)v * 8) = xv[j];
          }
          double sq = 0.0;
#pragma unroll
          for (int e = 0; e < 8; ++e) sq += (double)(x[e] * x[e]);  // x*x exact in fp32
          slot_add(ss, rr, sq);
        }
      }
      row_inv_rms(ss, rb, K, p.eps, red_d, stat);
      // ---- y = bf16(bf16(x inv) w)
#pragma unroll
      for (int j = 0; j < ITEMS; ++j) {
        const int i = threadIdx.x + j * NT;
        if (i < items) {
          const int rr = i / nvec;
          const float iv = stat[rr];
          float x[8], w[8];
          unpack8(xv[j], x);
          unpack8(wv[j], w);
          float m = 0.f;
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            x[e] = round_bf(round_bf(x[e] * iv) * w[e]);
            m = fmaxf(m, fabsf(x[e]));
          }
          xv[j] = pack8(x);
          slot_max(amax, rr, m);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < ITEMS; ++j) {
        const int i = threadIdx.x + j * NT;
        if (i < items) {
          const int rr = i / nvec, v = i - rr * nvec;
          xv[j] = __ldcg(reinterpret_cast<const uint4*>(p.x + (size_t)(r0 + rr) * K + (size_t)v * 8));
        }
      }
      if (!prefetched) {
        issue_prefetch();
        prefetched = true;
      }
      if (rowwise) {
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
          const int i = threadIdx.x + j * NT;
          if (i < items) {
            float x[8];
            unpack8(xv[j], x);
            float m = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(x[e]));
            slot_max(amax, i / nvec, m);
          }
        }
      }
    }
    // ---- scales and the e4m3 cast
    if (rowwise) {
      row_scales(amax, rb, red_f, stat);
      if ((int)threadIdx.x < rb) p.qscale[r0 + threadIdx.x] = stat[threadIdx.x];
    }
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
      const int i = threadIdx.x + j * NT;
      if (i < items) {
        const int rr = i / nvec, v = i - rr * nvec;
        float x[8];
        unpack8(xv[j], x);
        uint32_t lo = 0, hi = 0;
        if (rowwise) {
          const float sc = stat[rr], rcp = __frcp_rn(sc);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t bq = e4m3_quotient(x[e], sc, rcp);
            if (e < 4) lo |= bq << (8 * e);
            else hi |= bq << (8 * (e - 4));
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t bq = f2e4m3(clamp448(x[e] * p.inv));
            if (e < 4) lo |= bq << (8 * e);
            else hi |= bq << (8 * (e - 4));
          }
        }
        *reinterpret_cast<uint2*>(p.q8 + (size_t)(r0 + rr) * K + (size_t)v * 8) = make_uint2(lo, hi);
      }
    }
    __syncthreads();  // the next batch reuses the statistics in shared memory
  }
  if (!prefetched) issue_prefetch();
}

__device__ __forceinline__ void tile_coords(const GemmArgs& a, int t, int& tt, int& ks, int& ft) {
  tt = t % a.n_ttiles;
  const int rest = t / a.n_ttiles;
  ks = rest % a.splits;
  ft = rest / a.splits;
}
__device__ __forceinline__ void k_range(const GemmArgs& a, int ks, int nkb, int& kb0, int& kb1) {
  kb0 = (int)((long long)ks * nkb / a.splits);
  kb1 = (int)((long long)(ks + 1) * nkb / a.splits);
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}
__device__ __forceinline__ float lo_bf(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_bf(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Rotate-half RoPE of one token's normalised head, the quarter owned by this thread.
// xk holds packed bf16 pairs (elements 2i, 2i+1 in the low/high halves of a word) of head
// elements [16*PART, 16*PART + 16) in xk[0..8) and of their rotate-half partners
// [64 + 16*PART, 80 + 16*PART) in xk[8..16); inv = 1/rms of the whole head; cs holds this
// token's cos (cs[0..2)) and sin (cs[2..4)) at elements [16*PART, 16*PART + 16).  The
// tables' two halves are equal (rotate-half tables are cat(freqs, freqs)), so those values
// also serve the partners.  Writes the 32 outputs to dst (the 128-wide head row).
// Rounding as _legacy/lower_kernels.py:66-86: n = bf16(bf16(x * inv) * w), then
// y[e] = bf16(bf16(n[e] c) - bf16(n[e+64] s)), y[e+64] = bf16(bf16(n[e+64] c) + bf16(n[e] s)).
// Every product after the first is of two bf16 values, so the bf16x2 multiply (exact
// product, one rounding) and add (exact sum, one rounding) give those roundings exactly;
// the _rn forms keep the compiler from contracting a multiply and an add into one fma.
template <int PART>
__device__ __forceinline__ void qk_rope_part(const uint32_t (&xk)[16], float inv, const uint16_t* __restrict__ wn,
                                             const uint4 (&cs)[4], uint16_t* __restrict__ dst) {
  auto b2 = [](uint32_t w) { return *reinterpret_cast<const __nv_bfloat162*>(&w); };
  auto u32 = [](__nv_bfloat162 v) { return *reinterpret_cast<const uint32_t*>(&v); };
  // elements e and e+64 are rotate-half partners: handle 8 of each per step
#pragma unroll
  for (int r0 = 0; r0 < 16; r0 += 8) {
    const int e0 = 16 * PART + r0;
    const uint4 w0 = *reinterpret_cast<const uint4*>(wn + e0);
    const uint4 w1 = *reinterpret_cast<const uint4*>(wn + e0 + 64);
    const uint4 c0 = cs[r0 >> 3], s0 = cs[2 + (r0 >> 3)];
    const uint32_t wa[4] = {w0.x, w0.y, w0.z, w0.w}, wb[4] = {w1.x, w1.y, w1.z, w1.w};
    const uint32_t ca[4] = {c0.x, c0.y, c0.z, c0.w};
    const uint32_t sa[4] = {s0.x, s0.y, s0.z, s0.w};
    uint32_t ya[4], yb[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const uint32_t xa = xk[(r0 >> 1) + p], xb = xk[8 + (r0 >> 1) + p];  // elements e / e + 64
      const __nv_bfloat162 na = __hmul2_rn(__floats2bfloat162_rn(lo_bf(xa) * inv, hi_bf(xa) * inv), b2(wa[p]));
      const __nv_bfloat162 nb = __hmul2_rn(__floats2bfloat162_rn(lo_bf(xb) * inv, hi_bf(xb) * inv), b2(wb[p]));
      const __nv_bfloat162 c = b2(ca[p]), sn = b2(sa[p]);
      ya[p] = u32(__hadd2_rn(__hmul2_rn(na, c), __hmul2_rn(__hneg2(nb), sn)));  // y[e]    = n[e] c - n[e+64] s
      yb[p] = u32(__hadd2_rn(__hmul2_rn(nb, c), __hmul2_rn(na, sn)));           // y[e+64] = n[e+64] c + n[e] s
    }
    *reinterpret_cast<uint4*>(dst + e0) = make_uint4(ya[0], ya[1], ya[2], ya[3]);
    *reinterpret_cast<uint4*>(dst + e0 + 64) = make_uint4(yb[0], yb[1], yb[2], yb[3]);
  }
}

template <int BN, int EPI, int PRO>
__global__ void __launch_bounds__(threads_of(EPI), 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ CUtensorMap tmap_o, const GemmArgs args) {
  static_assert(EPI != EPI_QKROPE || BN == 128, "one head per tile");
  static_assert((EPI != FFB_EPI_SWIGLU && EPI != EPI_SWIGLU_Q8) || BN == 256, "gate/up pairs of 128 channels per tile");
  constexpr int EPI_WARPS = epi_warps(EPI);
  constexpr int BUFS = 16 / EPI_WARPS;  // staging buffers per epilogue warp
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stg_all = smem + C::STAGES * C::STAGE_BYTES;  // 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(stg_all + C::STG_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;  // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint64_t* xbar = tempty + 2;          // [4]: qkv epilogue, per lane quarter, 4 arrivals
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* sync_flag = reinterpret_cast<int*>(tmem_slot + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nkb = (args.K + BK - 1) / BK;

  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], EPI_WARPS);
    }
    for (int q = 0; q < 4; ++q) mbar_init(&xbar[q], 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_w);
    if (EPI != EPI_QKROPE) tma_prefetch_desc(&tmap_o);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // The weight half of the first ring pass does not depend on the previous kernel:
  // request it before the programmatic-launch wait -- or, with a fused prologue, right
  // after the prologue's own first loads (which would otherwise queue behind it).
  int pre = 0;
  auto prefetch_weights = [&]() {
    if (warp == 0 && lane == 0 && (int)blockIdx.x < args.n_tiles) {
      int tt, ks, ft, kb0, kb1;
      tile_coords(args, blockIdx.x, tt, ks, ft);
      k_range(args, ks, nkb, kb0, kb1);
      pre = kb1 - kb0 < C::STAGES ? kb1 - kb0 : C::STAGES;
      const uint64_t pol_w = policy_evict_first();
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
        tma_load_2d(smem + i * C::STAGE_BYTES + A_TILE_BYTES, &tmap_w, &full[i], (kb0 + i) * BK, ft * BN, pol_w);
      }
    }
  };
  if constexpr (PRO == PRO_NONE) prefetch_weights();
  if constexpr (PRO != PRO_NONE) {
    // Fused prologue: every CTA writes its slice of the A rows (and scales), then the grid
    // meets; the TMA loads of A below read rows other CTAs wrote.
    pdl_wait();
    prologue_rows<PRO>(args, stg_all, prefetch_weights);
    fence_proxy_async_global();  // this thread's rows, before the TMA loads of any CTA
    if (!grid_barrier(args.pro.sync, sync_flag)) {
      if (tid == 0) {
        *abort_flag = 1;
        atomicOr(&ffb_device_error_word, ffb::ERR_GRID_SYNC_TIMEOUT);
      }
      __syncthreads();
    }
  }

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first(), pol_a = policy_evict_last();
      pdl_wait();
      if (PRO != PRO_NONE) fence_proxy_async_global();  // the A rows other CTAs wrote, before the TMA reads them
      int it = 0;
      for (int t = blockIdx.x; t < args.n_tiles && !*abort_flag; t += gridDim.x) {
        int tt, ks, ft, kb0, kb1;
        tile_coords(args, t, tt, ks, ft);
        k_range(args, ks, nkb, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          uint8_t* st = smem + s * C::STAGE_BYTES;
          if (it < pre) {  // weight half already in flight
            tma_load_2d(st, &tmap_a, &full[s], kb * BK, tt * BM, pol_a);
            continue;
          }
          if (!mbar_wait_bounded(&empty[s], ((uint32_t)(it / C::STAGES) & 1u) ^ 1u, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_2d(st, &tmap_a, &full[s], kb * BK, tt * BM, pol_a);
          tma_load_2d(st + A_TILE_BYTES, &tmap_w, &full[s], kb * BK, ft * BN, pol_w);
        }
      }
      if (*abort_flag) {  // every slot whose copy was issued must land before the CTA exits
        volatile int never = 0;
        if (it < pre) {  // weight half requested, activation half not: request it so the slot completes
          int tt, ks, ft, kb0, kb1;
          tile_coords(args, blockIdx.x, tt, ks, ft);
          k_range(args, ks, nkb, kb0, kb1);
          for (int i = it; i < pre; ++i)
            tma_load_2d(smem + i * C::STAGE_BYTES, &tmap_a, &full[i], (kb0 + i) * BK, tt * BM, pol_a);
        }
        const int issued = it > pre ? it : pre;
        for (int i = (issued > C::STAGES ? issued - C::STAGES : 0); i < issued; ++i)
          mbar_wait_bounded(&full[i % C::STAGES], (uint32_t)(i / C::STAGES) & 1u, &never, 200000000ull);
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    pdl_wait();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3(BM, BN);
      int it = 0, lt = 0;
      for (int t = blockIdx.x; t < args.n_tiles && !*abort_flag; t += gridDim.x, ++lt) {
        int tt, ks, ft, kb0, kb1;
        tile_coords(args, t, tt, ks, ft);
        k_range(args, ks, nkb, kb0, kb1);
        const int buf = lt & 1;
        if (!mbar_wait_bounded(&tempty[buf], ((uint32_t)(lt >> 1) & 1u) ^ 1u, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * BN);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          if (!mbar_wait_bounded(&full[s], (uint32_t)(it / C::STAGES) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_u32(smem + s * C::STAGE_BYTES);
          const uint64_t da = umma_desc_sw128(base);
          const uint64_t dw = umma_desc_sw128(base + A_TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk)  // +32 bytes per K step = +2 encoded
            umma_f8f6f4(acc, da + 2 * kk, dw + 2 * kk, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        umma_commit(&tfull[buf]);  // fires when every MMA issued so far has completed
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    pdl_wait();
    if (warp == 2 && lane == 0) pdl_launch();
    const int q = warp & 3;            // TMEM lane quarter = this warp's 32 tokens
    const int half = (warp - 2) >> 2;  // which share of the tile's columns (0 .. EPI_WARPS/4 - 1)
    int lt = 0;
    uint32_t sc = 0;                   // staged-store counter (selects the staging buffer)
    for (int t = blockIdx.x; t < args.n_tiles; t += gridDim.x, ++lt) {
      int tt, ks, ft;
      tile_coords(args, t, tt, ks, ft);
      const int buf = lt & 1;
      const int m = tt * BM + q * 32 + lane;  // this thread's token
      const bool row_ok = m < args.M;
      const int n0 = ft * BN;
      // the tile's scales (and the RoPE tables of this thread's token) come from HBM / L2:
      // request them while the tile's MMAs run
      if (args.w_per_col && lane < BN / 32) prefetch_l1(args.w_scale + n0 + lane * 32);
      if (PRO == PRO_NONE && args.a_per_row && row_ok) prefetch_l1(args.a_scale + m);
      uint4 cs[4];  // qkv: this token's cos (loaded now) / sin (after the wait) at its 16 head elements
      if constexpr (EPI == EPI_QKROPE) {
        const RopeSide& r = args.rope;
        if (row_ok && ft < r.HQ + r.HK) {
          const uint4* cr = reinterpret_cast<const uint4*>(r.cos + (size_t)m * 128 + 16 * half);
          const uint4* sr = reinterpret_cast<const uint4*>(r.sin + (size_t)m * 128 + 16 * half);
          cs[0] = __ldg(cr);
          cs[1] = __ldg(cr + 1);
          prefetch_l1(sr);
          if (lane < 2) prefetch_l1((ft < r.HQ ? r.q_norm : r.k_norm) + 64 * lane);
        }
      }
      // each epilogue warp waits on its own; a timeout makes every one of them stop
      if (!(mbar_wait_bounded(&tfull[buf], (uint32_t)(lt >> 1) & 1u, abort_flag) && !*abort_flag)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      // (a fused prologue wrote the per-row scales in this kernel: read them from L2)
      const float sa = args.a_per_row ? (row_ok ? (PRO == PRO_NONE ? args.a_scale[m] : __ldcg(args.a_scale + m)) : 0.f)
                                      : args.a_scale[0];
      const uint32_t acc = tmem + (uint32_t)(buf * BN) + ((uint32_t)(q * 32) << 16);
      // per-feature scales of tile columns [c, c + 8)
      auto scales8 = [&](int c, float (&w)[8]) {
        if (args.w_per_col) {
          ldg8(args.w_scale + n0 + c, w);
        } else {
          const float w0 = args.w_scale[0];
#pragma unroll
          for (int j = 0; j < 8; ++j) w[j] = w0;
        }
      };

      if constexpr (EPI == EPI_QKROPE) {
        // One head per tile (BN == 128).  Warp share p of a lane quarter owns elements
        // [16p, 16p + 16) of each token's head and their rotate-half partners
        // [64 + 16p, 80 + 16p); the head's sum of squares (its RMSNorm statistic) is the
        // exact sum of the four shares' float64 partial sums, exchanged through shared memory.
        if (row_ok && ft < args.rope.HQ + args.rope.HK) {
          const uint4* sr = reinterpret_cast<const uint4*>(args.rope.sin + (size_t)m * 128 + 16 * half);
          cs[2] = __ldg(sr);
          cs[3] = __ldg(sr + 1);
        }
        uint32_t xk[16];
        double ssp = 0.0;
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const int c = 64 * g + 16 * half;
          uint32_t r[16];
          tmem_ld16_async(acc + (uint32_t)c, r);
          tmem_wait_ld();
          reg_fence(r);
#pragma unroll
          for (int j8 = 0; j8 < 16; j8 += 8) {
            float w[8];
            scales8(c + j8, w);
#pragma unroll
            for (int j = j8; j < j8 + 8; j += 2) {
              const uint32_t x2 = pack2(__uint_as_float(r[j]) * sa * w[j - j8], __uint_as_float(r[j + 1]) * sa * w[j - j8 + 1]);
              const float a = lo_bf(x2), b = hi_bf(x2);
              ssp += (double)(a * a) + (double)(b * b);  // x*x is exact in fp32 for bf16 x
              xk[8 * g + (j >> 1)] = x2;
            }
          }
        }
        // the store-staging area is unused by this epilogue: [2 tiles][4 shares][128 rows]
        double* slots = reinterpret_cast<double*>(stg_all) + (lt & 1) * 4 * BM;
        slots[half * BM + q * 32 + lane] = ssp;
        __syncwarp();
        if (lane == 0) mbar_arrive(&xbar[q]);
        if (!mbar_wait_bounded(&xbar[q], (uint32_t)lt & 1u, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        double ss = 0.0;
#pragma unroll
        for (int p = 0; p < 4; ++p) ss += slots[p * BM + q * 32 + lane];
        if (row_ok) {
          const RopeSide& r = args.rope;
          const size_t T = (size_t)args.M;
          if (ft < r.HQ + r.HK) {
            const bool is_q = ft < r.HQ;
            uint16_t* dst = is_q ? r.yq + ((size_t)ft * T + m) * 128 : r.yk + ((size_t)(ft - r.HQ) * T + m) * 128;
            const uint16_t* wn = is_q ? r.q_norm : r.k_norm;
            const float inv = inv_rms_from_ss(ss, 128, r.eps);
            switch (half) {
              case 0: qk_rope_part<0>(xk, inv, wn, cs, dst); break;
              case 1: qk_rope_part<1>(xk, inv, wn, cs, dst); break;
              case 2: qk_rope_part<2>(xk, inv, wn, cs, dst); break;
              default: qk_rope_part<3>(xk, inv, wn, cs, dst); break;
            }
          } else {  // v heads: copied through
            uint16_t* dst = r.yv + ((size_t)(ft - r.HQ - r.HK) * T + m) * 128 + half * 16;
            *reinterpret_cast<uint4*>(dst) = make_uint4(xk[0], xk[1], xk[2], xk[3]);
            *reinterpret_cast<uint4*>(dst + 8) = make_uint4(xk[4], xk[5], xk[6], xk[7]);
            *reinterpret_cast<uint4*>(dst + 64) = make_uint4(xk[8], xk[9], xk[10], xk[11]);
            *reinterpret_cast<uint4*>(dst + 72) = make_uint4(xk[12], xk[13], xk[14], xk[15]);
          }
        }
      } else {
        // Staged stores: the warp writes its [32 tokens x 64 B] chunk into one of its two
        // swizzled staging buffers and lane 0 issues a TMA store (rows >= M are clipped).
        auto staged_store = [&](const uint32_t (&w16)[16], int x, int z) {
          uint8_t* sb = stg_all + ((warp - 2) * BUFS + (int)(sc % BUFS)) * 2048;
          if (lane == 0) {  // the store that last used this buffer has read it
            if constexpr (BUFS == 2) bulk_wait_read<1>();
            else bulk_wait_read<0>();
          }
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 4; ++c)
            *reinterpret_cast<uint4*>(sb + lane * 64 + ((c ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(w16[4 * c], w16[4 * c + 1], w16[4 * c + 2], w16[4 * c + 3]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmap_o, sb, x, tt * BM + q * 32, z);
            bulk_commit();
          }
          ++sc;
        };
        // The same for a [32 tokens x 32 B] chunk of e4m3 bytes (unswizzled 32-byte rows).
        auto staged_store8 = [&](const uint32_t (&w8)[8], int x) {
          uint8_t* sb = stg_all + ((warp - 2) * BUFS + (int)(sc % BUFS)) * 2048;
          if (lane == 0) {
            if constexpr (BUFS == 2) bulk_wait_read<1>();
            else bulk_wait_read<0>();
          }
          __syncwarp();
          *reinterpret_cast<uint4*>(sb + lane * 32) = make_uint4(w8[0], w8[1], w8[2], w8[3]);
          *reinterpret_cast<uint4*>(sb + lane * 32 + 16) = make_uint4(w8[4], w8[5], w8[6], w8[7]);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&tmap_o, sb, x, tt * BM + q * 32, 0);
            bulk_commit();
          }
          ++sc;
        };
        if constexpr (EPI == FFB_EPI_SWIGLU || EPI == EPI_SWIGLU_Q8) {
          // columns [0, BN/2) are gate channels ft*BN/2 + j, [BN/2, BN) the matching up rows;
          // 8 channels at a time, the next group's TMEM loads in flight during the math.
          // EPI_SWIGLU_Q8 stores e4m3(clamp(bf16 output * out_inv, +-448)) instead: the static
          // FP8 quantisation of the down projection's input, done here instead of its own launch
          constexpr int HALFC = BN / 2;
          constexpr int PER_WARP = HALFC / (EPI_WARPS / 4);  // gate channels per warp
          const int cb = half * PER_WARP;
#pragma unroll 1
          for (int c0 = cb; c0 < cb + PER_WARP; c0 += 32) {
            uint32_t o[16];
            uint32_t o8[8];  // EPI_SWIGLU_Q8: 32 e4m3 bytes
            uint32_t g[2][8], u[2][8];
            tmem_ld8_async(acc + (uint32_t)c0, g[0]);
            tmem_ld8_async(acc + (uint32_t)(HALFC + c0), u[0]);
            tmem_wait_ld();
            reg_fence(g[0]);
            reg_fence(u[0]);
#pragma unroll
            for (int grp = 0; grp < 4; ++grp) {
              const int c = c0 + grp * 8, cur = grp & 1;
              if (grp < 3) {
                tmem_ld8_async(acc + (uint32_t)(c + 8), g[cur ^ 1]);
                tmem_ld8_async(acc + (uint32_t)(HALFC + c + 8), u[cur ^ 1]);
              }
              float wg[8], wu[8];
              scales8(c, wg);
              scales8(HALFC + c, wu);
              float act[8];  // bf16 SiLU of the bf16 gate values, looked up
#pragma unroll
              for (int j = 0; j < 8; ++j) act[j] = silu_lookup(round_bf(__uint_as_float(g[cur][j]) * sa * wg[j]));
#pragma unroll
              for (int j = 0; j < 8; j += 2) {
                float y2[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const float uv = round_bf(__uint_as_float(u[cur][j + h]) * sa * wu[j + h]);  // bf16 up
                  y2[h] = act[j + h] * uv;
                }
                if constexpr (EPI == EPI_SWIGLU_Q8) {
                  uint32_t qb = 0;
#pragma unroll
                  for (int h = 0; h < 2; ++h)
                    qb |= (uint32_t)f2e4m3(clamp448(round_bf(y2[h]) * args.out_inv)) << (8 * ((j + h) & 3));
                  if ((j & 3) == 0) o8[grp * 2 + (j >> 2)] = qb;
                  else o8[grp * 2 + (j >> 2)] |= qb;
                } else {
                  o[grp * 4 + (j >> 1)] = pack2(y2[0], y2[1]);
                }
              }
              if (grp < 3) {
                tmem_wait_ld();
                reg_fence(g[cur ^ 1]);
                reg_fence(u[cur ^ 1]);
              }
            }
            if constexpr (EPI == EPI_SWIGLU_Q8) staged_store8(o8, ft * HALFC + c0);
            else staged_store(o, ft * HALFC + c0, 0);
          }
        } else if constexpr (EPI == FFB_EPI_F32_PARTIAL) {
          constexpr int SHARE = BN / (EPI_WARPS / 4);  // columns per warp
#pragma unroll 1
          for (int c = half * SHARE; c < (half + 1) * SHARE; c += 16) {
            uint32_t r[16];
            tmem_ld16_async(acc + (uint32_t)c, r);
            float w0[8], w1[8];
            scales8(c, w0);
            scales8(c + 8, w1);
            tmem_wait_ld();
            reg_fence(r);
            uint32_t o[16];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              o[j] = __float_as_uint(__uint_as_float(r[j]) * sa * w0[j]);
              o[8 + j] = __float_as_uint(__uint_as_float(r[8 + j]) * sa * w1[j]);
            }
            staged_store(o, n0 + c, ks);
          }
        } else {
          constexpr int SHARE = BN / (EPI_WARPS / 4);  // columns per warp
#pragma unroll 1
          for (int c = half * SHARE; c < (half + 1) * SHARE; c += 32) {
            uint32_t r0[16], r1[16];
            tmem_ld16_async(acc + (uint32_t)c, r0);
            tmem_ld16_async(acc + (uint32_t)(c + 16), r1);
            tmem_wait_ld();
            reg_fence(r0);
            reg_fence(r1);
            uint32_t o[16];
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              float w[8];
              scales8(c + 8 * g, w);
              const uint32_t* r = g < 2 ? r0 : r1;
#pragma unroll
              for (int j = 0; j < 8; j += 2) {
                const int k = (g & 1) * 8 + j;
                o[g * 4 + (j >> 1)] = pack2(__uint_as_float(r[k]) * sa * w[j], __uint_as_float(r[k + 1]) * sa * w[j + 1]);
              }
            }
            staged_store(o, n0 + c, 0);
          }
        }
      }
      // this warp's TMEM reads of the buffer are complete (every tcgen05.ld waited): release it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    if (lane == 0) bulk_wait_all();  // every TMA store of this warp has landed
    __syncwarp();
  }

  if (warp == 1 && lane == 0 && *abort_flag) {
    // MMAs already issued must finish before their TMEM is released
    volatile int never = 0;
    mbar_wait_bounded(&tfull[0], 0, &never, 100000000ull);
    mbar_wait_bounded(&tfull[1], 0, &never, 100000000ull);
  }
  if (tid == 0 && *abort_flag) atomicOr(&ffb_device_error_word, ffb::ERR_GEMM_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

int num_sms() { return ffb::sm_count(); }

template <int BN, int EPI, int PRO>
cudaError_t launch_instance(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const GemmArgs& ga,
                            int grid, cudaStream_t stream) {
  using C = Cfg<BN>;
  cudaError_t ea = ffb::set_smem_attr(reinterpret_cast<const void*>(fp8_gemm_kernel<BN, EPI, PRO>), C::SMEM);
  if (ea != cudaSuccess) return ea;
  if constexpr (PRO != PRO_NONE) {
    // the fused prologue's grid barrier needs every CTA resident at once
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fp8_gemm_kernel<BN, EPI, PRO>,
                                                                  threads_of(EPI), C::SMEM);
    if (e != cudaSuccess) return e;
    if (grid > per_sm * num_sms()) return cudaErrorCooperativeLaunchTooLarge;
  }
  return ffb::launch(fp8_gemm_kernel<BN, EPI, PRO>, dim3(grid), dim3(threads_of(EPI)), C::SMEM, stream, ta, tw, to,
                     ga);
}

template <int BN, int PRO>
cudaError_t launch_epi(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const GemmArgs& ga,
                       int grid, cudaStream_t stream) {
  if constexpr (BN == 128) {
    if (ga.epilogue == EPI_QKROPE) return launch_instance<128, EPI_QKROPE, PRO>(ta, tw, to, ga, grid, stream);
    if (ga.epilogue == FFB_EPI_BF16) return launch_instance<128, FFB_EPI_BF16, PRO>(ta, tw, to, ga, grid, stream);
    if (ga.epilogue == FFB_EPI_F32_PARTIAL)
      return launch_instance<128, FFB_EPI_F32_PARTIAL, PRO>(ta, tw, to, ga, grid, stream);
  } else {
    if (ga.epilogue == FFB_EPI_SWIGLU) return launch_instance<256, FFB_EPI_SWIGLU, PRO>(ta, tw, to, ga, grid, stream);
    if constexpr (PRO == PRO_NONE)
      if (ga.epilogue == EPI_SWIGLU_Q8) return launch_instance<256, EPI_SWIGLU_Q8, PRO>(ta, tw, to, ga, grid, stream);
    if (ga.epilogue == FFB_EPI_BF16) return launch_instance<256, FFB_EPI_BF16, PRO>(ta, tw, to, ga, grid, stream);
    if (ga.epilogue == FFB_EPI_F32_PARTIAL)
      return launch_instance<256, FFB_EPI_F32_PARTIAL, PRO>(ta, tw, to, ga, grid, stream);
  }
  return cudaErrorInvalidValue;
}

template <int BN>
int launch_bn(const uint8_t* a8, const uint8_t* w8, GemmArgs& ga, int pro, cudaStream_t stream) {
  CUtensorMap ta, tw, to;
  memset(&to, 0, sizeof(to));
  int rc = ffb::make_tmap_2d(&ta, a8, (uint64_t)ga.M, (uint64_t)ga.K, (uint64_t)ga.K, BM, BK, 1);
  if (!rc) rc = ffb::make_tmap_2d(&tw, w8, (uint64_t)ga.N, (uint64_t)ga.K, (uint64_t)ga.K, BN, BK, 1);
  if (!rc && ga.epilogue == FFB_EPI_BF16)
    rc = ffb::make_tmap_out(&to, ga.out, 2, ga.N, ga.M, 1, (uint64_t)ga.N * 2, (uint64_t)ga.N * ga.M * 2, 32, 32);
  if (!rc && ga.epilogue == FFB_EPI_SWIGLU)
    rc = ffb::make_tmap_out(&to, ga.out, 2, ga.N / 2, ga.M, 1, (uint64_t)ga.N, (uint64_t)ga.N * ga.M, 32, 32);
  if (!rc && ga.epilogue == EPI_SWIGLU_Q8)
    rc = ffb::make_tmap_out(&to, ga.out, 1, ga.N / 2, ga.M, 1, (uint64_t)ga.N / 2, (uint64_t)ga.N / 2 * ga.M, 32, 32);
  if (!rc && ga.epilogue == FFB_EPI_F32_PARTIAL)
    rc = ffb::make_tmap_out(&to, ga.ws, 4, ga.N, ga.M, ga.splits, (uint64_t)ga.N * 4, (uint64_t)ga.N * ga.M * 4, 16,
                            32);
  if (rc) return rc;
  ga.n_ttiles = (ga.M + BM - 1) / BM;
  ga.n_tiles = (ga.N / BN) * ga.splits * ga.n_ttiles;
  const int grid = ga.n_tiles < num_sms() ? ga.n_tiles : num_sms();
  if (ga.epilogue == FFB_EPI_SWIGLU || ga.epilogue == EPI_SWIGLU_Q8) {
    rc = ffb::ensure_silu_table(stream);
    if (rc) return rc;
  }
  cudaError_t e = cudaErrorInvalidValue;
  if (pro == FFB_PRO_QUANT) e = launch_epi<BN, FFB_PRO_QUANT>(ta, tw, to, ga, grid, stream);
  else if (pro == FFB_PRO_ADD_RMSNORM) e = launch_epi<BN, FFB_PRO_ADD_RMSNORM>(ta, tw, to, ga, grid, stream);
  else e = launch_epi<BN, PRO_NONE>(ta, tw, to, ga, grid, stream);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_fp8_gemm: launch: %s", cudaGetErrorString(e));
  return FFB_OK;
}

int check_common(const uint8_t* a8, const float* a_scale, const uint8_t* w8, const float* w_scale, int M, int N,
                 int K) {
  FFB_REQUIRE(a8 && w8 && a_scale && w_scale, "ffb_fp8_gemm: NULL operand");
  FFB_REQUIRE(M > 0 && N > 0 && K > 0, "ffb_fp8_gemm: bad shape M=%d N=%d K=%d", M, N, K);
  FFB_REQUIRE(N % 128 == 0, "ffb_fp8_gemm: N=%d must be a multiple of 128", N);
  FFB_REQUIRE(K % 16 == 0, "ffb_fp8_gemm: K=%d must be a multiple of 16", K);
  FFB_REQUIRE(ffb::aligned(a8, 16) && ffb::aligned(w8, 16), "ffb_fp8_gemm: operands must be 16-byte aligned");
  FFB_REQUIRE(ffb::aligned(w_scale, 16), "ffb_fp8_gemm: w_scale must be 16-byte aligned");
  return FFB_OK;
}

// Validates the arguments of an FP8 GEMM and fills `ga`; returns the feature tile in bn.
int prep_gemm(GemmArgs& ga, int& bn, const uint8_t* a8, const float* a_scale, int a_per_row, const uint8_t* w8,
              const float* w_scale, int w_per_col, int epilogue, uint16_t* out, float* ws, int splits,
              int feature_tile, int M, int N, int K) {
  int rc = check_common(a8, a_scale, w8, w_scale, M, N, K);
  if (rc) return rc;
  FFB_REQUIRE(epilogue == FFB_EPI_BF16 || epilogue == FFB_EPI_F32_PARTIAL || epilogue == FFB_EPI_SWIGLU,
              "ffb_fp8_gemm: unknown epilogue %d", epilogue);
  const int nkb = (K + BK - 1) / BK;
  if (epilogue == FFB_EPI_F32_PARTIAL) {
    FFB_REQUIRE(ws != nullptr && ffb::aligned(ws, 16), "ffb_fp8_gemm: F32_PARTIAL needs a 16-byte aligned ws");
    FFB_REQUIRE(splits >= 1 && splits <= nkb, "ffb_fp8_gemm: splits=%d outside [1, %d]", splits, nkb);
  } else {
    FFB_REQUIRE(out != nullptr && ffb::aligned(out, 16), "ffb_fp8_gemm: out must be non-NULL, 16-byte aligned");
    FFB_REQUIRE(splits == 1, "ffb_fp8_gemm: splits must be 1 unless the epilogue is F32_PARTIAL");
  }
  bn = feature_tile > 0 ? feature_tile : (N % 256 == 0 ? 256 : 128);
  if (epilogue == FFB_EPI_SWIGLU) bn = 256;  // the gate/up interleave is per 128 channels
  FFB_REQUIRE(bn == 128 || bn == 256, "ffb_fp8_gemm: feature tile %d (128 or 256)", bn);
  FFB_REQUIRE(N % bn == 0, "ffb_fp8_gemm: N=%d must be a multiple of the feature tile %d", N, bn);
  ga = GemmArgs{};
  ga.a_scale = a_scale;
  ga.w_scale = w_scale;
  ga.out = out;
  ga.ws = ws;
  ga.a_per_row = a_per_row;
  ga.w_per_col = w_per_col;
  ga.epilogue = epilogue;
  ga.M = M;
  ga.N = N;
  ga.K = K;
  ga.splits = splits;
  return FFB_OK;
}

int prep_rope(GemmArgs& ga, const uint8_t* a8, const float* a_scale, int a_per_row, const uint8_t* w8,
              const float* w_scale, int w_per_col, const uint16_t* q_norm, const uint16_t* k_norm, float eps,
              const uint16_t* cos, const uint16_t* sin, uint16_t* yq, uint16_t* yk, uint16_t* yv, int T, int HQ,
              int HK, int K) {
  FFB_REQUIRE(HQ > 0 && HK > 0 && HQ % HK == 0, "ffb_fp8_gemm_qk_rope: bad heads HQ=%d HK=%d", HQ, HK);
  const int N = (HQ + 2 * HK) * 128;
  int rc = check_common(a8, a_scale, w8, w_scale, T, N, K);
  if (rc) return rc;
  FFB_REQUIRE(q_norm && k_norm && cos && sin && yq && yk && yv, "ffb_fp8_gemm_qk_rope: NULL pointer");
  FFB_REQUIRE(ffb::aligned(q_norm, 16) && ffb::aligned(k_norm, 16) && ffb::aligned(cos, 16) && ffb::aligned(sin, 16) &&
                  ffb::aligned(yq, 16) && ffb::aligned(yk, 16) && ffb::aligned(yv, 16),
              "ffb_fp8_gemm_qk_rope: 16-byte alignment");
  ga = GemmArgs{};
  ga.a_scale = a_scale;
  ga.w_scale = w_scale;
  ga.a_per_row = a_per_row;
  ga.w_per_col = w_per_col;
  ga.epilogue = EPI_QKROPE;
  ga.M = T;
  ga.N = N;
  ga.K = K;
  ga.splits = 1;
  ga.rope = RopeSide{q_norm, k_norm, cos, sin, yq, yk, yv, eps, HQ, HK};
  return FFB_OK;
}

// Validates a fused prologue and fills ga.pro (ga.M / ga.K already set).
int prep_prologue(GemmArgs& ga, const ffb_gemm_prologue* pro, uint8_t* a8, float* a_scale, int a_per_row) {
  FFB_REQUIRE(pro != nullptr, "ffb_fp8_gemm_fused: NULL prologue");
  FFB_REQUIRE(pro->kind == FFB_PRO_QUANT || pro->kind == FFB_PRO_ADD_RMSNORM, "ffb_fp8_gemm_fused: unknown kind %d",
              pro->kind);
  FFB_REQUIRE(pro->quant_mode == FFB_QUANT_STATIC || pro->quant_mode == FFB_QUANT_ROWWISE,
              "ffb_fp8_gemm_fused: quant_mode must be STATIC or ROWWISE");
  FFB_REQUIRE(a_per_row == (pro->quant_mode == FFB_QUANT_ROWWISE),
              "ffb_fp8_gemm_fused: a_per_row must be 1 exactly when quant_mode is ROWWISE");
  FFB_REQUIRE(pro->sync && ffb::aligned(pro->sync, 8), "ffb_fp8_gemm_fused: sync must be 8-byte aligned device words");
  FFB_REQUIRE(pro->x && ffb::aligned(pro->x, 16), "ffb_fp8_gemm_fused: x must be non-NULL, 16-byte aligned");
  const int K = ga.K, M = ga.M, NT = threads_of(0);
  FFB_REQUIRE(K % 8 == 0, "ffb_fp8_gemm_fused: K=%d must be a multiple of 8", K);
  FFB_REQUIRE(K / 8 <= pro_items(pro->kind) * NT, "ffb_fp8_gemm_fused: K=%d exceeds the prologue's %d", K,
              pro_items(pro->kind) * NT * 8);
  ProArgs& p = ga.pro;
  p = ProArgs{};
  p.x = pro->x;
  p.quant_mode = pro->quant_mode;
  p.inv = pro->inv_scale;
  p.q8 = a8;
  p.qscale = a_scale;
  p.sync = pro->sync;
  if (pro->kind == FFB_PRO_ADD_RMSNORM) {
    FFB_REQUIRE(pro->norm_w && ffb::aligned(pro->norm_w, 16), "ffb_fp8_gemm_fused: norm_w must be 16-byte aligned");
    p.w = pro->norm_w;
    p.eps = pro->eps;
    p.add = pro->add ? 1 : 0;
    if (p.add) {
      if (pro->b) {
        FFB_REQUIRE(ffb::aligned(pro->b, 16), "ffb_fp8_gemm_fused: b must be 16-byte aligned");
        p.b = pro->b;
      } else if (pro->b32) {
        FFB_REQUIRE(ffb::aligned(pro->b32, 16), "ffb_fp8_gemm_fused: b32 must be 16-byte aligned");
        FFB_REQUIRE(pro->splits >= 1 && pro->splits <= PRO_MAX_SPLITS, "ffb_fp8_gemm_fused: splits=%d outside [1, %d]",
                    pro->splits, PRO_MAX_SPLITS);
        p.b32 = pro->b32;
        p.splits = pro->splits;
      }
      FFB_REQUIRE(p.b || p.b32, "ffb_fp8_gemm_fused: add needs b or b32");
      if (pro->deep) {
        FFB_REQUIRE(ffb::aligned(pro->deep, 16), "ffb_fp8_gemm_fused: deep must be 16-byte aligned");
        FFB_REQUIRE(pro->start >= 0 && pro->nv >= 0 && pro->start + pro->nv <= M,
                    "ffb_fp8_gemm_fused: deep rows [%d, %d) outside [0, %d)", pro->start, pro->start + pro->nv, M);
        p.deep = pro->deep;
        p.start = pro->start;
        p.nv = pro->nv;
      }
      if (pro->residual) {
        FFB_REQUIRE(ffb::aligned(pro->residual, 16), "ffb_fp8_gemm_fused: residual must be 16-byte aligned");
        p.residual = pro->residual;
      }
    }
  }
  return FFB_OK;
}

}  // namespace

extern "C" int ffb_fp8_gemm(const uint8_t* a8, const float* a_scale, int a_per_row, const uint8_t* w8,
                            const float* w_scale, int w_per_col, int epilogue, uint16_t* out, float* ws, int splits,
                            int feature_tile, int M, int N, int K, void* stream) {
  GemmArgs ga;
  int bn = 0;
  const bool stream_tile = feature_tile == FFB_TILE_STREAM;
  int rc = prep_gemm(ga, bn, a8, a_scale, a_per_row, w8, w_scale, w_per_col, epilogue, out, ws, splits,
                     stream_tile ? 0 : feature_tile, M, N, K);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  FFB_REQUIRE(!stream_tile || ffb::stream_gemm_ctas(M, N, K, epilogue, splits) > 0,
              "ffb_fp8_gemm: the weight-stationary schedule does not apply (M=%d N=%d K=%d splits=%d: at most "
              "256 tokens per CTA and tiles x splits <= SMs)", M, N, K, splits);
  if (stream_tile || (feature_tile == 0 && splits == 1 && ffb::stream_gemm_preferred(M, N, K, epilogue)))
    return ffb::stream_gemm(a8, a_scale, a_per_row, w8, w_scale, w_per_col, epilogue,
                            epilogue == FFB_EPI_F32_PARTIAL ? static_cast<void*>(ws) : static_cast<void*>(out), splits,
                            0.f, nullptr, M, N, K, s);
  return bn == 256 ? launch_bn<256>(a8, w8, ga, PRO_NONE, s) : launch_bn<128>(a8, w8, ga, PRO_NONE, s);
}

extern "C" int ffb_fp8_gemm_swiglu_fp8(const uint8_t* a8, const float* a_scale, int a_per_row, const uint8_t* w8,
                                       const float* w_scale, int w_per_col, float out_inv, uint8_t* out8, int M,
                                       int N, int K, void* stream) {
  GemmArgs ga;
  int bn = 0;
  FFB_REQUIRE(out8 != nullptr && ffb::aligned(out8, 16), "ffb_fp8_gemm_swiglu_fp8: out8 must be 16-byte aligned");
  FFB_REQUIRE(out_inv > 0.f, "ffb_fp8_gemm_swiglu_fp8: out_inv must be positive");
  int rc = prep_gemm(ga, bn, a8, a_scale, a_per_row, w8, w_scale, w_per_col, FFB_EPI_SWIGLU,
                     reinterpret_cast<uint16_t*>(out8), nullptr, 1, 256, M, N, K);
  if (rc) return rc;
  ga.epilogue = EPI_SWIGLU_Q8;
  ga.out_inv = out_inv;
  if (ffb::stream_gemm_preferred(M, N, K, EPI_SWIGLU_Q8))
    return ffb::stream_gemm(a8, a_scale, a_per_row, w8, w_scale, w_per_col, EPI_SWIGLU_Q8, out8, 1, out_inv, nullptr,
                            M, N, K, reinterpret_cast<cudaStream_t>(stream));
  return launch_bn<256>(a8, w8, ga, PRO_NONE, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ffb_fp8_gemm_fused(const ffb_gemm_prologue* pro, uint8_t* a8, float* a_scale, int a_per_row,
                                  const uint8_t* w8, const float* w_scale, int w_per_col, int epilogue, uint16_t* out,
                                  float* ws, int splits, int feature_tile, int M, int N, int K, void* stream) {
  GemmArgs ga;
  int bn = 0;
  int rc = prep_gemm(ga, bn, a8, a_scale, a_per_row, w8, w_scale, w_per_col, epilogue, out, ws, splits, feature_tile,
                     M, N, K);
  if (!rc) rc = prep_prologue(ga, pro, a8, a_scale, a_per_row);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return bn == 256 ? launch_bn<256>(a8, w8, ga, pro->kind, s) : launch_bn<128>(a8, w8, ga, pro->kind, s);
}

extern "C" int ffb_fp8_gemm_qk_rope(const uint8_t* a8, const float* a_scale, int a_per_row, const uint8_t* w8,
                                    const float* w_scale, int w_per_col, const uint16_t* q_norm,
                                    const uint16_t* k_norm, float eps, const uint16_t* cos, const uint16_t* sin,
                                    uint16_t* yq, uint16_t* yk, uint16_t* yv, int T, int HQ, int HK, int K,
                                    void* stream) {
  GemmArgs ga;
  int rc = prep_rope(ga, a8, a_scale, a_per_row, w8, w_scale, w_per_col, q_norm, k_norm, eps, cos, sin, yq, yk, yv, T,
                     HQ, HK, K);
  if (rc) return rc;
  if (ffb::stream_gemm_preferred(T, ga.N, K, EPI_QKROPE))  // same field order as the stream kernel's block
    return ffb::stream_gemm(a8, a_scale, a_per_row, w8, w_scale, w_per_col, EPI_QKROPE, nullptr, 1, 0.f, &ga.rope, T,
                            ga.N, K, reinterpret_cast<cudaStream_t>(stream));
  return launch_bn<128>(a8, w8, ga, PRO_NONE, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ffb_fp8_gemm_qk_rope_fused(const ffb_gemm_prologue* pro, uint8_t* a8, float* a_scale, int a_per_row,
                                          const uint8_t* w8, const float* w_scale, int w_per_col,
                                          const uint16_t* q_norm, const uint16_t* k_norm, float eps,
                                          const uint16_t* cos, const uint16_t* sin, uint16_t* yq, uint16_t* yk,
                                          uint16_t* yv, int T, int HQ, int HK, int K, void* stream) {
  GemmArgs ga;
  int rc = prep_rope(ga, a8, a_scale, a_per_row, w8, w_scale, w_per_col, q_norm, k_norm, eps, cos, sin, yq, yk, yv, T,
                     HQ, HK, K);
  if (!rc) rc = prep_prologue(ga, pro, a8, a_scale, a_per_row);
  if (rc) return rc;
  return launch_bn<128>(a8, w8, ga, pro->kind, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int ffb_fp8_gemm_stream_ctas(int M, int N, int K, int epilogue, int splits) {
  if (epilogue != FFB_EPI_BF16 && epilogue != FFB_EPI_F32_PARTIAL && epilogue != FFB_EPI_SWIGLU) return 0;
  return ffb::stream_gemm_ctas(M, N, K, epilogue, splits);
}
