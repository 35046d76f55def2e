// FP8 e4m3 W8A8 linear for short token counts (prefill of a few hundred tokens) on the
// sm_100a tensor cores, "weight-stationary": the weight tile on the MMA's M side (128 output
// features), the tokens on N, and every CTA streaming exactly one weight tile.
//
// Why: at M = 320 tokens a token-major tile (128 tokens x 256 features) leaves the third
// token tile half empty, 228 tiles on 148 SMs make a second, one-third-full wave, and a
// split-K plan re-reads every weight tile once per token tile.  A CTA's mainloop costs
// ~70 ns per tcgen05.mma of its accumulator chain (measured on B200: nearly independent of
// N up to 256, and of the bytes per stage), i.e. ~0.28 us per 128-byte K block, so the
// plan wants one wave with the K blocks spread evenly; here each CTA gets one item: weight tile f (P = 2 tiles, gate and up, for
// SwiGLU), a range of 16-token units [u0, u0 + n) of the tile's tokens (C ranges per tile,
// n <= 16, so N = 16 n <= 256) and a range of K blocks (S splits; S > 1 writes fp32
// partial planes that the consumer sums).  G = tiles x C x S <= SMs: one wave, no CTA
// streams two tiles.  The C token ranges of a tile are neighbouring CTAs, so the tile
// crosses HBM about once.
//
// D^T[feature, token] accumulates in tensor memory (lane = feature, column = token).  Each
// output element is the same dot product over the same K range in the same K order as in
// the token-major kernel (gemm_fp8.cu), so the results are identical.
//
// Epilogues (the codes of gemm_fp8.cu): bf16 out [M, N]; fp32 split-K partial planes
// [S][M][N]; SwiGLU (out [M, N/2] bf16, or with static scales e4m3 bytes for the down
// projection); qkv + per-head QK RMSNorm + rotate-half M-RoPE (one head per weight tile)
// through a shared-memory transpose.  The epilogue is latency-bound (a few units of 16
// tokens per warp), so everything it reads that does not depend on the accumulators (the
// per-token scales, the norm weights, the rotary rows) is requested before it waits, and
// the bf16 / fp32 outputs leave as direct row-segment stores (no staging round trip).
//
// Roles (576 threads): warp 0 TMA producer (the weight tile(s) + one [16 n x 128 B] token
// box per stage; the weight half of the first stages is requested before the programmatic-
// launch wait); warp 1 TMEM allocator + single-thread MMA issuer; warps 2..17 epilogue
// (warp % 4 = TMEM lane quarter = 32 features, (warp - 2) / 4 = share of the units).  Every
// wait is bounded; a timeout sets the abort flag and the device error word.
#include "common.cuh"
#include "pdl.cuh"

#include <string.h>

namespace {

constexpr int FT = 128;          // output features per weight tile (UMMA M)
constexpr int UN = 16;           // tokens per work unit (UMMA N granule; one TMA box)
constexpr int BK = 128;          // K bytes per stage (one 128-byte swizzle row)
constexpr int A_TILE = FT * BK;  // 16 KB
constexpr int B_UNIT = UN * BK;  // 2 KB
constexpr int MAXSTAGES = 8;
constexpr int EPI_WARPS = 16;
constexpr int THREADS = 64 + EPI_WARPS * 32;
constexpr int SMEM_LIMIT = 232448;
constexpr int STG_BYTES = 32768;  // epilogue staging: 16 warps x 2 KB, or 4 shares x 2 x 4 KB
constexpr int BAR_BYTES = 512;
constexpr int FIXED = STG_BYTES + BAR_BYTES + 1024;

// epilogue codes (as gemm_fp8.cu)
constexpr int E_BF16 = FFB_EPI_BF16;
constexpr int E_F32 = FFB_EPI_F32_PARTIAL;
constexpr int E_SWIGLU = FFB_EPI_SWIGLU;
constexpr int E_QKROPE = 100;
constexpr int E_SWIGLU_Q8 = 101;

struct StreamRope {
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

struct StreamArgs {
  const float* a_scale;
  const float* w_scale;
  int a_per_row, w_per_col;
  int M, N, K;
  int P;          // weight tiles per item: 2 (gate, up) for SwiGLU, else 1
  int NU, C, S;   // token units; token ranges per tile; K splits
  int b_bytes;    // token bytes per stage (max units per CTA x 2 KB)
  int stages;
  uint32_t tmem_cols;
  float out_inv;  // E_SWIGLU_Q8: static inverse scale of the next linear's input
  void* out;      // E_BF16 / E_F32: the output (stored directly, one 128 / 64-byte row segment per warp store)
  StreamRope rope;
};

// The item of CTA b: token ranges fastest (the C CTAs of one weight tile run together).
struct Item {
  int f, u0, n, kb0, kb1;  // weight tile; first unit and units; K blocks [kb0, kb1)
};
__host__ __device__ inline Item cta_item(int b, int NU, int C, int S, int nkb) {
  const int tr = b % C, ks = (b / C) % S, f = b / (C * S);
  Item it;
  it.f = f;
  it.u0 = tr * NU / C;
  it.n = (tr + 1) * NU / C - it.u0;
  it.kb0 = ks * nkb / S;
  it.kb1 = (ks + 1) * nkb / S;
  return it;
}

__device__ __forceinline__ float lo_of(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float hi_of(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    fp8_gemm_stream_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                           const __grid_constant__ CUtensorMap tmap_o, const StreamArgs args) {
  constexpr int P = (EPI == E_SWIGLU || EPI == E_SWIGLU_Q8) ? 2 : 1;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int stage_bytes = P * A_TILE + args.b_bytes;  // a multiple of 2 KB
  uint8_t* stg = smem + args.stages * stage_bytes;     // 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(stg + STG_BYTES);
  uint64_t* empty = full + MAXSTAGES;
  uint64_t* tfull = empty + MAXSTAGES;
  uint64_t* xbar = tfull + 1;  // [4] qkv epilogue: per share, 4 warp arrivals per unit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(xbar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nkb = (args.K + BK - 1) / BK;
  const Item item = cta_item(blockIdx.x, args.NU, args.C, args.S, nkb);
  const int n = item.n, nk = item.kb1 - item.kb0;
  const int ks = (blockIdx.x / args.C) % args.S;

  if (tid == 0) {
    for (int s = 0; s < args.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&xbar[i], 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_w);
    if (EPI == E_SWIGLU || EPI == E_SWIGLU_Q8) tma_prefetch_desc(&tmap_o);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, args.tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first(), pol_a = policy_evict_last();
      const int wrow = item.f * P * FT, trow = item.u0 * UN;
      // the weight tiles of the first ring pass do not depend on the previous kernel
      const int pre = nk < args.stages ? nk : args.stages;
      for (int i = 0; i < pre; ++i) {
        uint8_t* st = smem + i * stage_bytes;
        mbar_arrive_expect_tx(&full[i], P * A_TILE + args.b_bytes);
#pragma unroll
        for (int p = 0; p < P; ++p)
          tma_load_2d(st + p * A_TILE, &tmap_w, &full[i], (item.kb0 + i) * BK, wrow + p * FT, pol_w);
      }
      pdl_wait();
      int it = 0, s = 0;
      uint32_t ph = 0;  // phase of the ring pass (kept incrementally: no division in the loop)
      for (int kb = item.kb0; kb < item.kb1 && !*abort_flag; ++kb, ++it) {
        uint8_t* st = smem + s * stage_bytes;
        if (it >= pre) {
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[s], P * A_TILE + args.b_bytes);
#pragma unroll
          for (int p = 0; p < P; ++p)
            tma_load_2d(st + p * A_TILE, &tmap_w, &full[s], kb * BK, wrow + p * FT, pol_w);
        }
        // one box of the largest unit range: rows past this CTA's range (or past M) are
        // loaded and never read
        tma_load_2d(st + P * A_TILE, &tmap_a, &full[s], kb * BK, trow, pol_a);
        if (++s == args.stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (*abort_flag) {  // every slot whose copy was issued must land before the CTA exits
        volatile int never = 0;
        for (int j = it; j < pre; ++j)  // requested before the wait, never given their tokens
          tma_load_2d(smem + j * stage_bytes + P * A_TILE, &tmap_a, &full[j], (item.kb0 + j) * BK, trow, pol_a);
        const int issued = it > pre ? it : pre;
        for (int j = (issued > args.stages ? issued - args.stages : 0); j < issued; ++j)
          mbar_wait_bounded(&full[j % args.stages], (uint32_t)(j / args.stages) & 1u, &never, 200000000ull);
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    pdl_wait();
    if (lane == 0) {
      // one MMA per K step and weight tile, N = 16 n; the issuing thread's loop carries no
      // division and no memory access besides the waits
      const uint32_t idesc = idesc_e4m3(FT, n * UN);
      const uint32_t smem_base = smem_u32(smem);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int kb = item.kb0; kb < item.kb1; ++kb) {
        if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = smem_base + (uint32_t)(s * stage_bytes);
        const uint64_t da0 = umma_desc_sw128(base);
        const uint64_t db0 = umma_desc_sw128(base + P * A_TILE);
#pragma unroll
        for (int kk = 0; kk < BK / 32; ++kk) {
#pragma unroll
          for (int p = 0; p < P; ++p)
            umma_f8f6f4(tmem + (uint32_t)(p * n * UN), da0 + (uint64_t)(p * (A_TILE >> 4)) + 2 * kk, db0 + 2 * kk,
                        idesc, (kb > item.kb0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty[s]);
        if (++s == args.stages) {
          s = 0;
          ph ^= 1u;
        }
      }
      umma_commit(tfull);  // fires when every MMA issued has completed (also after a failed wait)
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    pdl_wait();
    if (warp == 2 && lane == 0) pdl_launch();
    const int q = warp & 3;             // TMEM lane quarter: features [32q, 32q + 32) of the tile
    const int share = (warp - 2) >> 2;  // units share, 0..3
    const int fl = q * 32 + lane;       // this thread's feature in the tile
    const int f = item.f;
    uint32_t sc = 0;                    // staged stores issued by this warp
    int xu = 0;                         // qkv: units processed by this share (buffer parity)
    bool ok = true;
    // per-feature weight scales of this thread's row(s)
    float sw0 = 0.f, sw1 = 0.f;
    if (args.w_per_col) {
      sw0 = __ldg(args.w_scale + (size_t)(f * P) * FT + fl);
      if (P == 2) sw1 = __ldg(args.w_scale + (size_t)(f * P + 1) * FT + fl);
    } else {
      sw0 = sw1 = __ldg(args.w_scale);
    }
    // this warp's activation scales, requested while the MMAs run: unit share + 4 i (i < 4,
    // n <= 16), token j of it sits in lane 16 (i & 1) + j of sreg[i >> 1]; tokens past M
    // get 0
    float sreg[2] = {0.f, 0.f};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int u = share + 4 * (2 * h + (lane >> 4)), t = (item.u0 + u) * UN + (lane & 15);
      if (!args.a_per_row)
        sreg[h] = __ldg(args.a_scale);
      else if (u < n && t < args.M)
        sreg[h] = __ldg(args.a_scale + t);
    }
    // qkv: the RMSNorm weights of this thread's 8 + 8 elements (part lane & 7 of every token)
    uint4 wn0 = make_uint4(0u, 0u, 0u, 0u), wn1 = wn0;
    if constexpr (EPI == E_QKROPE) {
      if (f < args.rope.HQ + args.rope.HK) {
        const uint16_t* wn = f < args.rope.HQ ? args.rope.q_norm : args.rope.k_norm;
        wn0 = __ldg(reinterpret_cast<const uint4*>(wn + 8 * (lane & 7)));
        wn1 = __ldg(reinterpret_cast<const uint4*>(wn + 64 + 8 * (lane & 7)));
      }
    }
    if (!mbar_wait_bounded(tfull, 0u, abort_flag)) ok = false;
    tc_fence_after();
    const uint32_t acc = tmem + ((uint32_t)(q * 32) << 16);
    for (int u = share, i = 0; u < n && ok; u += 4, ++i) {
      const int t0 = (item.u0 + u) * UN;  // first token of the unit
      float sa[UN];
      const float sv = (i >> 1) ? sreg[1] : sreg[0];
#pragma unroll
      for (int j = 0; j < UN; ++j) sa[j] = __shfl_sync(0xffffffffu, sv, ((i & 1) << 4) + j);
      uint32_t r0[16];
      tmem_ld16_async(acc + (uint32_t)(u * UN), r0);
      if constexpr (P == 2) {
        uint32_t r1[16];
        tmem_ld16_async(acc + (uint32_t)(n * UN + u * UN), r1);
        tmem_wait_ld();
        reg_fence(r0);
        reg_fence(r1);
        uint8_t* sb = stg + ((warp - 2) * 2 + (int)(sc & 1)) * 1024;
        if (lane == 0) bulk_wait_read<1>();  // the store that last used this buffer has read it
        __syncwarp();
#pragma unroll
        for (int j = 0; j < UN; ++j) {
          const float act = silu_lookup(round_bf(__uint_as_float(r0[j]) * sa[j] * sw0));  // bf16 SiLU of bf16 gate
          const float up = round_bf(__uint_as_float(r1[j]) * sa[j] * sw1);
          const float y = act * up;
          if constexpr (EPI == E_SWIGLU_Q8)
            sb[j * 32 + lane] = f2e4m3(clamp448(round_bf(y) * args.out_inv));
          else
            *reinterpret_cast<uint16_t*>(sb + j * 64 + lane * 2) = f2bf(y);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&tmap_o, sb, (EPI == E_SWIGLU_Q8 ? 1 : 2) * (f * FT + q * 32), t0);
          bulk_commit();
        }
        ++sc;
      } else if constexpr (EPI == E_BF16) {
        // one 64-byte row segment (32 features) per token and store
        tmem_wait_ld();
        reg_fence(r0);
        uint16_t* dst = reinterpret_cast<uint16_t*>(args.out) + (size_t)t0 * args.N + f * FT + fl;
#pragma unroll
        for (int j = 0; j < UN; ++j)
          if (t0 + j < args.M) dst[(size_t)j * args.N] = f2bf(__uint_as_float(r0[j]) * sa[j] * sw0);
      } else if constexpr (EPI == E_F32) {
        // this K split's fp32 partial (acc * sa * sw), plane ks of [S][M][N]: one 128-byte
        // row segment per token and store
        tmem_wait_ld();
        reg_fence(r0);
        float* dst = reinterpret_cast<float*>(args.out) + ((size_t)ks * args.M + t0) * args.N + f * FT + fl;
#pragma unroll
        for (int j = 0; j < UN; ++j)
          if (t0 + j < args.M) dst[(size_t)j * args.N] = __uint_as_float(r0[j]) * sa[j] * sw0;
      } else {
        // qkv: (1) the 4 warps of this share write the unit's bf16 head rows into a
        // [16 tokens x 128 features] tile; (2) the same 128 threads, 8 per token, each
        // normalise and rotate 8 elements and their rotate-half partners (+64).  The
        // rotary rows of step (2) are requested first, so they arrive during step (1).
        const StreamRope& r = args.rope;
        const int idx = q * 32 + lane, jt = idx >> 3, pp = idx & 7;  // token jt of the unit, part pp
        const int t = t0 + jt;
        const bool qk_row = f < r.HQ + r.HK && t < args.M;
        uint4 c0 = make_uint4(0u, 0u, 0u, 0u), s0 = c0;
        if (qk_row) {
          c0 = __ldg(reinterpret_cast<const uint4*>(r.cos + (size_t)t * 128 + 8 * pp));
          s0 = __ldg(reinterpret_cast<const uint4*>(r.sin + (size_t)t * 128 + 8 * pp));
        }
        tmem_wait_ld();
        reg_fence(r0);
        uint8_t* xt = stg + (share * 2 + (xu & 1)) * 4096;
#pragma unroll
        for (int j = 0; j < UN; ++j)
          *reinterpret_cast<uint16_t*>(xt + j * 256 + fl * 2) = f2bf(__uint_as_float(r0[j]) * sa[j] * sw0);
        __syncwarp();
        if (lane == 0) mbar_arrive(&xbar[share]);
        if (!mbar_wait_bounded(&xbar[share], (uint32_t)xu & 1u, abort_flag)) {
          ok = false;
          break;
        }
        ++xu;
        const uint4 xa = *reinterpret_cast<const uint4*>(xt + jt * 256 + pp * 16);        // elements 8pp..
        const uint4 xb = *reinterpret_cast<const uint4*>(xt + jt * 256 + 128 + pp * 16);  // elements 64+8pp..
        const uint32_t wa[4] = {xa.x, xa.y, xa.z, xa.w}, wb[4] = {xb.x, xb.y, xb.z, xb.w};
        const size_t T = (size_t)args.M;
        if (f >= r.HQ + r.HK) {  // v heads: copied through
          if (t < args.M) {
            uint16_t* dst = r.yv + ((size_t)(f - r.HQ - r.HK) * T + t) * 128;
            *reinterpret_cast<uint4*>(dst + 8 * pp) = xa;
            *reinterpret_cast<uint4*>(dst + 64 + 8 * pp) = xb;
          }
        } else {
          double ss = 0.0;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float a0 = lo_of(wa[e]), a1 = hi_of(wa[e]), b0 = lo_of(wb[e]), b1 = hi_of(wb[e]);
            ss += (double)(a0 * a0) + (double)(a1 * a1) + (double)(b0 * b0) + (double)(b1 * b1);  // exact squares
          }
          ss += __shfl_xor_sync(0xffffffffu, ss, 1);
          ss += __shfl_xor_sync(0xffffffffu, ss, 2);
          ss += __shfl_xor_sync(0xffffffffu, ss, 4);
          if (qk_row) {
            const bool is_q = f < r.HQ;
            uint16_t* dst = is_q ? r.yq + ((size_t)f * T + t) * 128 : r.yk + ((size_t)(f - r.HQ) * T + t) * 128;
            const float inv = inv_rms_from_ss(ss, 128, r.eps);
            const uint32_t wna[4] = {wn0.x, wn0.y, wn0.z, wn0.w}, wnb[4] = {wn1.x, wn1.y, wn1.z, wn1.w};
            const uint32_t ca[4] = {c0.x, c0.y, c0.z, c0.w}, sa4[4] = {s0.x, s0.y, s0.z, s0.w};
            auto b2 = [](uint32_t w) { return *reinterpret_cast<const __nv_bfloat162*>(&w); };
            auto u32 = [](__nv_bfloat162 v) { return *reinterpret_cast<const uint32_t*>(&v); };
            uint32_t ya[4], yb[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              // n = bf16(bf16(x inv) w); y[e] = bf16(bf16(n[e] c) - bf16(n[e+64] s)),
              // y[e+64] = bf16(bf16(n[e+64] c) + bf16(n[e] s))  (_legacy/lower_kernels.py:66-86)
              const __nv_bfloat162 na =
                  __hmul2_rn(__floats2bfloat162_rn(lo_of(wa[e]) * inv, hi_of(wa[e]) * inv), b2(wna[e]));
              const __nv_bfloat162 nb =
                  __hmul2_rn(__floats2bfloat162_rn(lo_of(wb[e]) * inv, hi_of(wb[e]) * inv), b2(wnb[e]));
              const __nv_bfloat162 c = b2(ca[e]), sn = b2(sa4[e]);
              ya[e] = u32(__hadd2_rn(__hmul2_rn(na, c), __hmul2_rn(__hneg2(nb), sn)));
              yb[e] = u32(__hadd2_rn(__hmul2_rn(nb, c), __hmul2_rn(na, sn)));
            }
            *reinterpret_cast<uint4*>(dst + 8 * pp) = make_uint4(ya[0], ya[1], ya[2], ya[3]);
            *reinterpret_cast<uint4*>(dst + 64 + 8 * pp) = make_uint4(yb[0], yb[1], yb[2], yb[3]);
          }
        }
      }
    }
    if (!ok) *abort_flag = 1;
    // this warp's TMEM reads are complete (every tcgen05.ld waited); its stores land
    tc_fence_before();
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  if (warp == 1 && lane == 0 && *abort_flag) {
    // MMAs already issued must finish before their TMEM is released (the issuer committed
    // them to tfull)
    volatile int never = 0;
    mbar_wait_bounded(tfull, 0, &never, 100000000ull);
  }
  if (tid == 0 && *abort_flag) atomicOr(&ffb_device_error_word, ffb::ERR_GEMM_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, args.tmem_cols);
  }
}

}  // namespace

namespace ffb {

// Plans the weight-stationary schedule of an M x N x K GEMM with P weight tiles per item and
// S K splits on the current device: C token ranges per weight tile, as many as one wave of
// SMs allows (fewer tokens per CTA, fewer bytes per K block).  Returns false when no C fits
// (a CTA would hold more than 16 units = 256 tokens, or the tiles x S items alone exceed
// the SMs, or fewer than two pipeline stages fit).
static bool stream_plan(int M, int N, int K, int P, int S, StreamArgs& a, int& grid) {
  if (M <= 0 || N % (FT * P) != 0 || S < 1) return false;
  const int nkb = (K + BK - 1) / BK;
  if (S > nkb) return false;
  a.NU = (M + UN - 1) / UN;
  const int NF = N / (FT * P);
  const int sms = sm_count();
  if (NF * S > sms) return false;
  int C = sms / (NF * S);
  if (C > a.NU) C = a.NU;
  const int max_units = (a.NU + C - 1) / C;
  if (max_units > 16) return false;  // N = 16 n <= 256; also the TMA box height
  a.C = C;
  a.S = S;
  grid = NF * C * S;
  a.b_bytes = max_units * B_UNIT;
  const int stage = P * A_TILE + a.b_bytes;
  int stages = (SMEM_LIMIT - FIXED) / stage;
  if (stages > MAXSTAGES) stages = MAXSTAGES;
  if (stages < 2) return false;
  a.stages = stages;
  uint32_t cols = 32;
  while (cols < (uint32_t)(P * max_units * UN)) cols <<= 1;
  a.tmem_cols = cols;
  return true;
}

static int epi_tiles(int epilogue) { return (epilogue == E_SWIGLU || epilogue == E_SWIGLU_Q8) ? 2 : 1; }

int stream_gemm_ctas(int M, int N, int K, int epilogue, int splits) {
  if (epilogue != E_BF16 && epilogue != E_F32 && epilogue != E_SWIGLU && epilogue != E_SWIGLU_Q8 &&
      epilogue != E_QKROPE)
    return 0;
  if (splits != 1 && epilogue != E_F32) return 0;
  StreamArgs a = {};
  int grid = 0;
  return stream_plan(M, N, K, epi_tiles(epilogue), splits, a, grid) ? grid : 0;
}

// The automatic choice (feature_tile 0, and the qkv / static-SwiGLU entries): the weight-
// stationary schedule up to 512 tokens when it applies; above, 128-token tiles are full and
// fill the machine.
bool stream_gemm_preferred(int M, int N, int K, int epilogue) {
  return M <= 512 && stream_gemm_ctas(M, N, K, epilogue, 1) > 0;
}

template <int EPI>
static int launch_stream(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const StreamArgs& a,
                         int grid, cudaStream_t stream) {
  const int P = (EPI == E_SWIGLU || EPI == E_SWIGLU_Q8) ? 2 : 1;
  const int smem = a.stages * (P * A_TILE + a.b_bytes) + FIXED;
  cudaError_t e = set_smem_attr(reinterpret_cast<const void*>(fp8_gemm_stream_kernel<EPI>), smem);
  if (e == cudaSuccess)
    e = launch(fp8_gemm_stream_kernel<EPI>, dim3(grid), dim3(THREADS), (size_t)smem, stream, ta, tw, to, a);
  if (e != cudaSuccess) return fail(FFB_ECUDA, "ffb_fp8_gemm (weight-stationary): launch: %s", cudaGetErrorString(e));
  return FFB_OK;
}

// The weight-stationary GEMM (argument checks are the caller's).  out: bf16 [M, N]
// (E_BF16), fp32 [splits][M][N] (E_F32), bf16 [M, N/2] (E_SWIGLU), e4m3 [M, N/2]
// (E_SWIGLU_Q8); rope_side: E_QKROPE's argument block.
int stream_gemm(const uint8_t* a8, const float* a_scale, int a_per_row, const uint8_t* w8, const float* w_scale,
                int w_per_col, int epilogue, void* out, int splits, float out_inv, const void* rope_side, int M, int N,
                int K, cudaStream_t stream) {
  StreamArgs a = {};
  int grid = 0;
  const int P = epi_tiles(epilogue);
  if (stream_gemm_ctas(M, N, K, epilogue, splits) == 0 || !stream_plan(M, N, K, P, splits, a, grid))
    return fail(FFB_EINVAL, "ffb_fp8_gemm: the weight-stationary schedule does not apply to M=%d N=%d K=%d splits=%d",
                M, N, K, splits);
  a.a_scale = a_scale;
  a.w_scale = w_scale;
  a.a_per_row = a_per_row;
  a.w_per_col = w_per_col;
  a.M = M;
  a.N = N;
  a.K = K;
  a.P = P;
  a.out_inv = out_inv;
  a.out = out;
  if (rope_side) memcpy(&a.rope, rope_side, sizeof(StreamRope));
  CUtensorMap ta, tw, to;
  memset(&to, 0, sizeof(to));
  int rc = make_tmap_2d(&ta, a8, (uint64_t)M, (uint64_t)K, (uint64_t)K, (uint32_t)(a.b_bytes / BK), BK, 1);
  if (!rc) rc = make_tmap_2d(&tw, w8, (uint64_t)N, (uint64_t)K, (uint64_t)K, FT, BK, 1);
  // SwiGLU outputs through unswizzled [16 rows x 64 B] (bf16) or [16 x 32 B] (e4m3) boxes
  if (!rc && epilogue == E_SWIGLU)
    rc = make_tmap_2d_bytes(&to, out, (uint64_t)M, (uint64_t)N, (uint64_t)N, UN, 64);
  if (!rc && epilogue == E_SWIGLU_Q8)
    rc = make_tmap_2d_bytes(&to, out, (uint64_t)M, (uint64_t)N / 2, (uint64_t)N / 2, UN, 32);
  if (rc) return rc;
  if (epilogue == E_SWIGLU || epilogue == E_SWIGLU_Q8) {
    rc = ensure_silu_table(stream);
    if (rc) return rc;
  }
  switch (epilogue) {
    case E_BF16: return launch_stream<E_BF16>(ta, tw, to, a, grid, stream);
    case E_F32: return launch_stream<E_F32>(ta, tw, to, a, grid, stream);
    case E_SWIGLU: return launch_stream<E_SWIGLU>(ta, tw, to, a, grid, stream);
    case E_SWIGLU_Q8: return launch_stream<E_SWIGLU_Q8>(ta, tw, to, a, grid, stream);
    case E_QKROPE: return launch_stream<E_QKROPE>(ta, tw, to, a, grid, stream);
    default: return fail(FFB_EINVAL, "ffb_fp8_gemm: epilogue %d has no weight-stationary form", epilogue);
  }
}

}  // namespace ffb
