// bf16 linear with bias on the sm_100a tensor cores (tcgen05.mma kind::f16, fp32
// accumulators in tensor memory), for the vision tower in front of the language path:
// patch embedding, qkv / proj / fc1 / fc2 of every block and the mergers' two linears.
//
// Replaces the nn.Linear / Conv3d calls of the reference's vision wrappers
// (_legacy/vision_graph_runtime.py:16-27 runs the HF blocks; scaled_qwen_runtime.py:42-55,
// `NativeNormVision.core`): y = bf16(x W^T + b) with the bias added to the fp32
// accumulator, and the operations the blocks apply to that bf16 output folded into the
// epilogue: the residual add (bf16(res + y)) and the activations (bf16(gelu(y)), tanh
// form in the blocks' MLP, erf form in the mergers).
//
// Tile = 128 tokens (UMMA M) x BN output features (UMMA N = 64, 128 or 256), 64 K
// elements (one 128-byte swizzle row of bf16) per stage.  Persistent kernel, one CTA per
// SM, tiles round-robin with the token tile fastest (CTAs that run at the same time share
// weight tiles in L2).  Roles (64 + 32 x EW threads; EW = 16 epilogue warps for BN >= 128,
// 8 for BN = 64):
//   warp 0      TMA producer: activation tile [128 x 64] and weight tile [BN x 64], both
//               K-major with the 128-byte swizzle, into a ring of STAGES slots; the first
//               ring pass of weight tiles is requested before the wait on the previous
//               kernel (weights do not depend on it);
//   warp 1      TMEM allocator + single-thread MMA issuer (4 x K16 per stage) into one of
//               two accumulators, so the epilogue of tile i overlaps the mainloop of i+1;
//   warps 2..   epilogue: lane quarter (warp % 4) x one of EW / 4 column groups; 32
//               columns at a time: fp32 accumulator + bias, the epilogue's operation,
//               bf16, staged in shared memory and written by TMA store (rows past M and
//               columns past N are clipped by the store).  With one or two tiles per CTA
//               the last tile's epilogue is exposed, so the GELU epilogues get 16 warps.
// K past the end of the operands is zero-filled by TMA (adds nothing), so K need not be
// a multiple of 64.  Every wait is bounded; a timeout sets the abort flag and the device
// error word, and TMEM is released.
#include "common.cuh"
#include "pdl.cuh"

namespace {

constexpr int BM = 128;
constexpr int BKE = 64;
constexpr int UMMA_K = 16;
constexpr int A_BYTES = BM * BKE * 2;  // 16 KB
constexpr int SMEM_LIMIT = 232448;

template <int BN>
struct BCfg {
  static constexpr int EW = BN >= 128 ? 16 : 8;  // epilogue warps
  static constexpr int NSTG = EW == 16 ? 1 : 2;  // 2 KB staging buffers per epilogue warp
  static constexpr int THREADS = 64 + EW * 32;
  static constexpr int W_BYTES = BN * BKE * 2;
  static constexpr int STAGE_BYTES = A_BYTES + W_BYTES;
  static constexpr int STG_BYTES = EW * NSTG * 2048;
  static constexpr int FIXED = STG_BYTES + 512 + 1024;
  static constexpr int FIT = (SMEM_LIMIT - FIXED) / STAGE_BYTES;
  static constexpr int STAGES = FIT > 8 ? 8 : FIT;
  static constexpr int SMEM = STAGES * STAGE_BYTES + FIXED;
  static constexpr int TMEM_COLS = 2 * BN;
  static_assert(BN == 64 || BN == 128 || BN == 256, "feature tile 64, 128 or 256");
  static_assert(STAGE_BYTES % 1024 == 0, "swizzled tiles need 1024-byte alignment");
};

struct BArgs {
  const uint16_t* bias;  // [N] bf16 or NULL (no bias)
  const uint16_t* res;   // [M][N] bf16 (FFB_EPI_BIAS_RES)
  uint16_t* out;         // [M][N] bf16 (the cluster split-K kernel's direct stores)
  float* ws;             // split-K: [splits][M][N] fp32 partial planes
  uint32_t* counters;    // split-K: arrivals per output tile (zero between launches)
  int M, N, K, n_ttiles, n_tiles, splits;
};

// Tile t -> token tile (fastest), K split, feature tile; the split's K blocks [kb0, kb1).
__device__ __forceinline__ void tile_coords(const BArgs& a, int t, int nkb, int& tt, int& ks, int& ft, int& kb0,
                                            int& kb1) {
  tt = t % a.n_ttiles;
  const int r = t / a.n_ttiles;
  ks = r % a.splits;
  ft = r / a.splits;
  kb0 = (int)((long long)ks * nkb / a.splits);
  kb1 = (int)((long long)(ks + 1) * nkb / a.splits);
}

// Both GELU forms are (x / 2) s with s = 1 + tanh(u) or 1 + erf(z), and s is evaluated
// without the cancellation of 1 + (a value near -1): for u, z < 0 it is the small
// positive term itself.  IEEE-rounded fp32 operations only (restated in oracle/act.c).
//
// tanh form: u = 0.7978845608 (x + 0.044715 x^3); with r = 2 / (e^(2|u|) + 1) (e by
// exp2_poly of fp32(|u| 2 log2 e); r = 0 from |u| >= 40 on), s = r for u < 0, 2 - r
// otherwise.  Absolute error of s below 1e-6.  r is computed as 2 * (1 / d) with the
// reciprocal correctly rounded: equal to the correctly rounded 2 / d, because scaling by 2
// is exact (d = e + 1 lies in [2, 2^117), so neither product nor reciprocal leaves the
// normal range), and a reciprocal is cheaper than a general IEEE divide.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float x3 = __fmul_rn(__fmul_rn(x, x), x);
  const float u = __fmul_rn(0.797884560802865355f, __fadd_rn(x, __fmul_rn(0.044715f, x3)));
  const float a = fabsf(u);
  float r = 0.f;
  if (!(a >= 40.f)) r = __fmul_rn(2.f, __frcp_rn(__fadd_rn(exp2_poly(__fmul_rn(a, 2.88539008177792681f)), 1.f)));
  const float s = u < 0.f ? r : __fsub_rn(2.f, r);
  return __fmul_rn(__fmul_rn(0.5f, x), s);
}
// erf form: z = x / sqrt 2; erfc(|z|) ~ q = t (a1 + t (a2 + t (a3 + t (a4 + t a5))))
// e^(-z^2), t = 1 / (1 + p |z|) (Abramowitz & Stegun 7.1.26, |error| <= 1.5e-7; Horner with
// fused multiply-adds; e^(-z^2) by exp2_poly of fp32(fp32(z^2) * -log2 e)); s = q for
// z < 0, 2 - q otherwise.  (1 / (1 + p|z|) is the correctly rounded reciprocal.)
__device__ __forceinline__ float gelu_erf(float x) {
  const float z = __fmul_rn(x, 0.707106781186547524f);
  const float a = fabsf(z);
  const float t = __frcp_rn(__fadd_rn(1.f, __fmul_rn(0.3275911f, a)));
  float p = 1.061405429f;
  p = __fmaf_rn(p, t, -1.453152027f);
  p = __fmaf_rn(p, t, 1.421413741f);
  p = __fmaf_rn(p, t, -0.284496736f);
  p = __fmaf_rn(p, t, 0.254829592f);
  p = __fmul_rn(p, t);
  const float q = __fmul_rn(p, exp2_poly(__fmul_rn(__fmul_rn(a, a), -1.44269504088896341f)));
  const float s = z < 0.f ? q : __fsub_rn(2.f, q);
  return __fmul_rn(__fmul_rn(x, 0.5f), s);
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}
__device__ __forceinline__ void unpack8(uint4 v, float* f) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

template <int EPI>
__device__ __forceinline__ float epilogue_op(float acc, float b, float r) {
  const float v = __fadd_rn(acc, b);
  if constexpr (EPI == FFB_EPI_BIAS) return v;
  if constexpr (EPI == FFB_EPI_BIAS_RES) return __fadd_rn(r, round_bf(v));
  if constexpr (EPI == FFB_EPI_BIAS_GELU_TANH) return gelu_tanh(round_bf(v));
  return gelu_erf(round_bf(v));
}

template <int BN, int EPI>
__global__ void __launch_bounds__(BCfg<BN>::THREADS, 1)
    bf16_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                     const __grid_constant__ CUtensorMap tmap_o, const BArgs args) {
  using C = BCfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stg_all = smem + C::STAGES * C::STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(stg_all + C::STG_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;  // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_flag = abort_flag + 1;  // split-K: the epilogue warps' shared verdict per tile

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nkb = (args.K + BKE - 1) / BKE;

  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], C::EW);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_o);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
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
      int pre = 0, tt0 = 0, kb00 = 0;
      if ((int)blockIdx.x < args.n_tiles) {  // weights do not depend on the previous kernel
        int ks, ft, kb1;
        tile_coords(args, blockIdx.x, nkb, tt0, ks, ft, kb00, kb1);
        pre = kb1 - kb00 < C::STAGES ? kb1 - kb00 : C::STAGES;
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
          tma_load_2d(smem + i * C::STAGE_BYTES + A_BYTES, &tmap_w, &full[i], (kb00 + i) * BKE, ft * BN, pol_w);
        }
      }
      pdl_wait();
      int it = 0, s = 0;
      uint32_t ph = 0;
      for (int t = blockIdx.x; t < args.n_tiles && !*abort_flag; t += gridDim.x) {
        int tt, ks, ft, kb0, kb1;
        tile_coords(args, t, nkb, tt, ks, ft, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          uint8_t* st = smem + s * C::STAGE_BYTES;
          if (it >= pre) {
            if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
              *abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
            tma_load_2d(st + A_BYTES, &tmap_w, &full[s], kb * BKE, ft * BN, pol_w);
          }
          tma_load_2d(st, &tmap_a, &full[s], kb * BKE, tt * BM, pol_a);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
      if (*abort_flag) {  // every slot whose copy was issued must land before the CTA exits
        volatile int never = 0;
        for (int j = it; j < pre; ++j)  // requested before the wait, never given their activations
          tma_load_2d(smem + j * C::STAGE_BYTES, &tmap_a, &full[j], (kb00 + j) * BKE, tt0 * BM, pol_a);
        const int issued = it > pre ? it : pre;
        for (int j = (issued > C::STAGES ? issued - C::STAGES : 0); j < issued; ++j)
          mbar_wait_bounded(&full[j % C::STAGES], (uint32_t)(j / C::STAGES) & 1u, &never, 200000000ull);
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    pdl_wait();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN);
      const uint32_t smem_base = smem_u32(smem);
      int s = 0, lt = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < args.n_tiles && ok; t += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (!mbar_wait_bounded(&tempty[buf], ((uint32_t)(lt >> 1) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * BN);
        int tt, ks, ft, kb0, kb1;
        tile_coords(args, t, nkb, tt, ks, ft, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t base = smem_base + (uint32_t)(s * C::STAGE_BYTES);
          const uint64_t da = umma_desc_sw128(base);
          const uint64_t dw = umma_desc_sw128(base + A_BYTES);
#pragma unroll
          for (int kk = 0; kk < BKE / UMMA_K; ++kk)  // +32 bytes per K step = +2 encoded
            umma_f16(acc, da + 2 * kk, dw + 2 * kk, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
          if (++s == C::STAGES) {
            s = 0;
            ph ^= 1u;
          }
        }
        umma_commit(&tfull[buf]);  // fires when this tile's MMAs (or all issued) complete
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    pdl_wait();
    if (warp == 2 && lane == 0) pdl_launch();
    const int q = warp & 3;             // TMEM lane quarter = this warp's 32 tokens
    constexpr int GROUP = BN / (C::EW / 4);  // columns per column group
    const int cg = (warp - 2) >> 2;          // this warp's column group
    int lt = 0;
    uint32_t sc = 0;
    for (int t = blockIdx.x; t < args.n_tiles; t += gridDim.x, ++lt) {
      int tt, ks, ft, kb0, kb1;
      tile_coords(args, t, nkb, tt, ks, ft, kb0, kb1);
      const int buf = lt & 1;
      const bool got = mbar_wait_bounded(&tfull[buf], (uint32_t)(lt >> 1) & 1u, abort_flag) && !*abort_flag;
      if (!got) *abort_flag = 1;
      tc_fence_after();
      const uint32_t acc = tmem + (uint32_t)(buf * BN) + ((uint32_t)(q * 32) << 16);
      const int row = tt * BM + q * 32 + lane;  // this thread's token
      const bool rows_in = tt * BM + q * 32 < args.M;  // warp-uniform
      if (args.splits > 1) {
        // split-K: every split writes its fp32 partial plane; the split that arrives last
        // at the tile's counter sums the planes in split order and runs the epilogue.  All
        // epilogue warps take both named barriers on every tile (also after a failed wait)
        // and leave together on the verdict thread 0 of warp 2 publishes between them.
        if (got && rows_in) {
#pragma unroll 1
          for (int c = cg * GROUP; c < (cg + 1) * GROUP; c += 32) {
            const int n = ft * BN + c;
            if (n >= args.N) continue;
            uint32_t r[32];
            tmem_ld16_async(acc + (uint32_t)c, *reinterpret_cast<uint32_t(*)[16]>(r));
            tmem_ld16_async(acc + (uint32_t)(c + 16), *reinterpret_cast<uint32_t(*)[16]>(r + 16));
            tmem_wait_ld();
            reg_fence(r);
            if (row < args.M) {
              float* dst = args.ws + ((size_t)ks * args.M + row) * args.N + n;
#pragma unroll
              for (int g = 0; g < 4; ++g)
                if (n + 8 * g < args.N) {
                  reinterpret_cast<uint4*>(dst + 8 * g)[0] = make_uint4(r[8 * g], r[8 * g + 1], r[8 * g + 2], r[8 * g + 3]);
                  reinterpret_cast<uint4*>(dst + 8 * g)[1] =
                      make_uint4(r[8 * g + 4], r[8 * g + 5], r[8 * g + 6], r[8 * g + 7]);
                }
            }
          }
        }
        __threadfence();
        named_barrier(1, C::EW * 32);
        if (warp == 2 && lane == 0) {
          int verdict = -1;  // -1: stop (a wait gave up somewhere); 0: not last; 1: last
          if (!*abort_flag) {
            const int tile_out = tt + args.n_ttiles * ft;
            const uint32_t old = atomicAdd(args.counters + tile_out, 1u);
            verdict = old == (uint32_t)(args.splits - 1) ? 1 : 0;
            if (verdict) args.counters[tile_out] = 0;  // every split has arrived: ready for the next launch
          }
          *last_flag = verdict;
        }
        named_barrier(1, C::EW * 32);
        const int verdict = *last_flag;
        if (verdict < 0) break;
        if (verdict == 0) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&tempty[buf]);
          continue;
        }
        __threadfence();  // the other splits' planes, published before their arrivals
      } else if (!got) {
        break;
      }
#pragma unroll 1
      for (int c = cg * GROUP; c < (cg + 1) * GROUP; c += 32) {
        const int n = ft * BN + c;  // first output feature of the chunk
        // chunks wholly past N or past M store nothing (warp-uniform: n and q are)
        if (n >= args.N || !rows_in) continue;
        uint32_t r0[16], r1[16];
        tmem_ld16_async(acc + (uint32_t)c, r0);
        tmem_ld16_async(acc + (uint32_t)(c + 16), r1);
        float bv[32], rv[32];
#pragma unroll
        for (int g = 0; g < 4; ++g) {  // N is a multiple of 8: a group is all in or all out
          const bool in = n + 8 * g < args.N;
          const uint4 z = make_uint4(0, 0, 0, 0);
          unpack8(args.bias && in ? __ldg(reinterpret_cast<const uint4*>(args.bias + n + 8 * g)) : z, bv + 8 * g);
          if constexpr (EPI == FFB_EPI_BIAS_RES)
            unpack8(in && row < args.M ? *reinterpret_cast<const uint4*>(args.res + (size_t)row * args.N + n + 8 * g)
                                       : z,
                    rv + 8 * g);
        }
        tmem_wait_ld();
        reg_fence(r0);
        reg_fence(r1);
        if (args.splits > 1 && row < args.M) {
          // total = ((p0 + p1) + p2) + ...: this split's own partial from TMEM, the others'
          // from their planes (L2, bypassing L1); four columns at a time
          const float* srcp = args.ws + (size_t)row * args.N + n;
          const size_t plane = (size_t)args.M * args.N;
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            uint32_t* rg = g < 4 ? r0 + 4 * g : r1 + 4 * (g - 4);
            if (n + 4 * g >= args.N) continue;
            float4 t4 = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
            for (int j = 0; j < args.splits; ++j) {
              const float4 p4 = j == ks ? make_float4(__uint_as_float(rg[0]), __uint_as_float(rg[1]),
                                                      __uint_as_float(rg[2]), __uint_as_float(rg[3]))
                                        : __ldcg(reinterpret_cast<const float4*>(srcp + j * plane) + g);
              if (j == 0) {
                t4 = p4;
              } else {
                t4.x = __fadd_rn(t4.x, p4.x);
                t4.y = __fadd_rn(t4.y, p4.y);
                t4.z = __fadd_rn(t4.z, p4.z);
                t4.w = __fadd_rn(t4.w, p4.w);
              }
            }
            rg[0] = __float_as_uint(t4.x);
            rg[1] = __float_as_uint(t4.y);
            rg[2] = __float_as_uint(t4.z);
            rg[3] = __float_as_uint(t4.w);
          }
        }
        uint32_t o[16];
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          o[j >> 1] = pack2(epilogue_op<EPI>(__uint_as_float(r0[j]), bv[j], rv[j]),
                            epilogue_op<EPI>(__uint_as_float(r0[j + 1]), bv[j + 1], rv[j + 1]));
          o[8 + (j >> 1)] = pack2(epilogue_op<EPI>(__uint_as_float(r1[j]), bv[16 + j], rv[16 + j]),
                                  epilogue_op<EPI>(__uint_as_float(r1[j + 1]), bv[17 + j], rv[17 + j]));
        }
        // 32 rows x 64 bytes, 64-byte swizzle (make_tmap_out), NSTG buffers per warp
        uint8_t* sb = stg_all + ((warp - 2) * C::NSTG + (int)(sc % C::NSTG)) * 2048;
        if (lane == 0) bulk_wait_read<C::NSTG - 1>();  // the store that last used this buffer has read it
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *reinterpret_cast<uint4*>(sb + lane * 64 + ((k ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&tmap_o, sb, n, tt * BM + q * 32, 0);
          bulk_commit();
        }
        ++sc;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  if (warp == 1 && lane == 0 && *abort_flag) {
    // MMAs already issued must finish before their TMEM and shared memory are released
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

// ---------------------------------------------------------------------------------------
// Cluster split-K (`bf16_gemm_cluster_kernel`): one [128 x 256] output tile per cluster of
// CS CTAs (CS = 2 or 4); cluster rank r computes K split r.  A CTA's mainloop costs about
// the same per tcgen05.mma whatever its N (the single accumulator chain is latency-bound),
// so 256-wide tiles do 4x the work of 64-wide ones per instruction; at the vision tower's
// shapes (M = 1024 tokens, N = 1024) there are only 32 such tiles, and the K split puts them
// on 128 SMs.  After its MMAs each CTA writes its fp32 partial into its own shared memory
// (the drained stage ring, 128 KB, 16-byte chunks XOR-swizzled by row so that a warp's
// stores and its peers' reads are bank-conflict free); one cluster barrier; CTA r then sums
// rows [r 128/CS, (r+1) 128/CS) of the CS partials in split order over distributed shared
// memory (((p0 + p1) + p2) + p3, the order of the plane path and of the oracle), applies the
// epilogue and stores its rows as coalesced 8-byte bf16 groups; a second cluster barrier
// keeps every partial alive until each peer has read it.  Every CTA takes both barriers on
// every path (a timeout sets the error word and leaves the output undefined).
constexpr int CTHREADS = 64 + 16 * 32;
template <int EPI, int CS>
__global__ void __launch_bounds__(CTHREADS, 1)
    bf16_gemm_cluster_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                             const BArgs args) {
  using C = BCfg<256>;
  constexpr int BN = 256;
  constexpr int RING = C::STAGES * C::STAGE_BYTES;
  static_assert(RING >= BM * BN * 4, "the fp32 partial reuses the stage ring");
  static_assert(C::THREADS == CTHREADS, "16 epilogue warps");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + RING);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* part = reinterpret_cast<float*>(smem);  // [128 rows][64 chunks of 4], chunk c of row at (c ^ (row & 7))

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rank = (int)cluster_ctarank();
  const int tile = (int)blockIdx.x / CS;
  const int tt = tile % args.n_ttiles, ft = tile / args.n_ttiles;
  const int nkb = (args.K + BKE - 1) / BKE;
  const int kb0 = (int)((long long)rank * nkb / CS), kb1 = (int)((long long)(rank + 1) * nkb / CS);
  const int nk = kb1 - kb0;

  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, BN);
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
      const int pre = nk < C::STAGES ? nk : C::STAGES;
      for (int i = 0; i < pre; ++i) {  // weights do not depend on the previous kernel
        mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
        tma_load_2d(smem + i * C::STAGE_BYTES + A_BYTES, &tmap_w, &full[i], (kb0 + i) * BKE, ft * BN, pol_w);
      }
      pdl_wait();
      int it = 0, s = 0;
      uint32_t ph = 0;
      for (int kb = kb0; kb < kb1 && !*abort_flag; ++kb, ++it) {
        uint8_t* st = smem + s * C::STAGE_BYTES;
        if (it >= pre) {
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_2d(st + A_BYTES, &tmap_w, &full[s], kb * BKE, ft * BN, pol_w);
        }
        tma_load_2d(st, &tmap_a, &full[s], kb * BKE, tt * BM, pol_a);
        if (++s == C::STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (*abort_flag) {  // every slot whose copy was issued must land before the ring is reused
        volatile int never = 0;
        for (int j = it; j < pre; ++j)
          tma_load_2d(smem + j * C::STAGE_BYTES, &tmap_a, &full[j], (kb0 + j) * BKE, tt * BM, pol_a);
        const int issued = it > pre ? it : pre;
        for (int j = (issued > C::STAGES ? issued - C::STAGES : 0); j < issued; ++j)
          mbar_wait_bounded(&full[j % C::STAGES], (uint32_t)(j / C::STAGES) & 1u, &never, 200000000ull);
      }
    } else {
      pdl_wait();
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    pdl_wait();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_bf16(BM, BN);
      const uint32_t smem_base = smem_u32(smem);
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = smem_base + (uint32_t)(s * C::STAGE_BYTES);
        const uint64_t da = umma_desc_sw128(base);
        const uint64_t dw = umma_desc_sw128(base + A_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKE / UMMA_K; ++kk)
          umma_f16(tmem, da + 2 * kk, dw + 2 * kk, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[s]);
        if (++s == C::STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
      umma_commit(tfull);  // fires when every MMA issued has completed (also after a failed wait)
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------------------ partial -> own shared memory
    pdl_wait();
    if (warp == 2 && lane == 0) pdl_launch();
    const int q = warp & 3, cg = (warp - 2) >> 2;  // lane quarter (32 rows), 64-column group
    const int row = q * 32 + lane;
    if (!(mbar_wait_bounded(tfull, 0u, abort_flag) && !*abort_flag)) *abort_flag = 1;
    tc_fence_after();
    if (!*abort_flag) {
      const uint32_t acc = tmem + ((uint32_t)(q * 32) << 16);
      float4* prow = reinterpret_cast<float4*>(part + row * BN);
#pragma unroll 1
      for (int c = cg * 64; c < cg * 64 + 64; c += 32) {
        uint32_t r0[16], r1[16];
        tmem_ld16_async(acc + (uint32_t)c, r0);
        tmem_ld16_async(acc + (uint32_t)(c + 16), r1);
        tmem_wait_ld();
        reg_fence(r0);
        reg_fence(r1);
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // 16-byte chunks c / 4 + j of this row
          const uint32_t* rr = j < 4 ? r0 + 4 * j : r1 + 4 * (j - 4);
          prow[((c >> 2) + j) ^ (row & 7)] = make_float4(__uint_as_float(rr[0]), __uint_as_float(rr[1]),
                                                         __uint_as_float(rr[2]), __uint_as_float(rr[3]));
        }
      }
    }
    tc_fence_before();
  }

  cluster_sync();  // every partial of the cluster is in its CTA's shared memory

  if (warp >= 2) {
    // ------------------------------------------------------------------ reduce this rank's rows
    constexpr int RPC = BM / CS;  // rows per cluster rank
    const int et = tid - 64;
    uint32_t peer[CS];
#pragma unroll
    for (int p = 0; p < CS; ++p) peer[p] = cluster_map(part, (uint32_t)p);
#pragma unroll 1
    for (int i = et; i < RPC * 64; i += 16 * 32) {
      const int rl = rank * RPC + (i >> 6), c = i & 63;  // tile row, 16-byte chunk (4 columns)
      const int m = tt * BM + rl, n = ft * BN + 4 * c;
      if (m >= args.M || n >= args.N) continue;
      const uint32_t off = (uint32_t)((rl * 64 + (c ^ (rl & 7))) * 16);
      float4 t = ld_cluster_f4(peer[0] + off);
#pragma unroll
      for (int p = 1; p < CS; ++p) {
        const float4 v = ld_cluster_f4(peer[p] + off);
        t.x = __fadd_rn(t.x, v.x);
        t.y = __fadd_rn(t.y, v.y);
        t.z = __fadd_rn(t.z, v.z);
        t.w = __fadd_rn(t.w, v.w);
      }
      float bv[4] = {0.f, 0.f, 0.f, 0.f}, rv[4] = {0.f, 0.f, 0.f, 0.f};
      if (args.bias) {
        const uint2 b2 = __ldg(reinterpret_cast<const uint2*>(args.bias + n));
        bv[0] = __uint_as_float(b2.x << 16);
        bv[1] = __uint_as_float(b2.x & 0xFFFF0000u);
        bv[2] = __uint_as_float(b2.y << 16);
        bv[3] = __uint_as_float(b2.y & 0xFFFF0000u);
      }
      if constexpr (EPI == FFB_EPI_BIAS_RES) {
        const uint2 r2 = *reinterpret_cast<const uint2*>(args.res + (size_t)m * args.N + n);
        rv[0] = __uint_as_float(r2.x << 16);
        rv[1] = __uint_as_float(r2.x & 0xFFFF0000u);
        rv[2] = __uint_as_float(r2.y << 16);
        rv[3] = __uint_as_float(r2.y & 0xFFFF0000u);
      }
      const uint2 o = make_uint2(pack2(epilogue_op<EPI>(t.x, bv[0], rv[0]), epilogue_op<EPI>(t.y, bv[1], rv[1])),
                                 pack2(epilogue_op<EPI>(t.z, bv[2], rv[2]), epilogue_op<EPI>(t.w, bv[3], rv[3])));
      *reinterpret_cast<uint2*>(args.out + (size_t)m * args.N + n) = o;
    }
  }

  cluster_sync();  // no CTA leaves while a peer may still read its partial

  if (warp == 1 && lane == 0 && *abort_flag) {
    volatile int never = 0;  // MMAs already issued must finish before TMEM is released
    mbar_wait_bounded(tfull, 0, &never, 100000000ull);
  }
  if (tid == 0 && *abort_flag) atomicOr(&ffb_device_error_word, ffb::ERR_GEMM_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, BN);
  }
}

template <int BN, int EPI>
cudaError_t launch_instance(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const BArgs& ba,
                            int grid, cudaStream_t stream) {
  using C = BCfg<BN>;
  cudaError_t e = ffb::set_smem_attr(reinterpret_cast<const void*>(bf16_gemm_kernel<BN, EPI>), C::SMEM);
  if (e != cudaSuccess) return e;
  return ffb::launch(bf16_gemm_kernel<BN, EPI>, dim3(grid), dim3(C::THREADS), C::SMEM, stream, ta, tw, to, ba);
}

template <int EPI, int CS>
cudaError_t launch_cluster_instance(const CUtensorMap& ta, const CUtensorMap& tw, const BArgs& ba, int grid,
                                   cudaStream_t stream) {
  using C = BCfg<256>;
  constexpr int SMEM = C::STAGES * C::STAGE_BYTES + 256 + 1024;
  cudaError_t e = ffb::set_smem_attr(reinterpret_cast<const void*>(bf16_gemm_cluster_kernel<EPI, CS>), SMEM);
  if (e != cudaSuccess) return e;
  return ffb::launch_cluster(bf16_gemm_cluster_kernel<EPI, CS>, dim3(grid), dim3(CTHREADS), SMEM, CS, stream, ta, tw,
                             ba);
}

template <int CS>
cudaError_t launch_cluster_epi(int epilogue, const CUtensorMap& ta, const CUtensorMap& tw, const BArgs& ba, int grid,
                               cudaStream_t stream) {
  switch (epilogue) {
    case FFB_EPI_BIAS: return launch_cluster_instance<FFB_EPI_BIAS, CS>(ta, tw, ba, grid, stream);
    case FFB_EPI_BIAS_RES: return launch_cluster_instance<FFB_EPI_BIAS_RES, CS>(ta, tw, ba, grid, stream);
    case FFB_EPI_BIAS_GELU_TANH: return launch_cluster_instance<FFB_EPI_BIAS_GELU_TANH, CS>(ta, tw, ba, grid, stream);
    default: return launch_cluster_instance<FFB_EPI_BIAS_GELU_ERF, CS>(ta, tw, ba, grid, stream);
  }
}

// The cluster kernel serves 256-wide tiles split 2 or 4 ways (one CTA per split).
bool cluster_split(int bn, int splits) { return bn == 256 && (splits == 2 || splits == 4); }

template <int BN>
cudaError_t launch_epi(int epilogue, const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to,
                       const BArgs& ba, int grid, cudaStream_t stream) {
  switch (epilogue) {
    case FFB_EPI_BIAS: return launch_instance<BN, FFB_EPI_BIAS>(ta, tw, to, ba, grid, stream);
    case FFB_EPI_BIAS_RES: return launch_instance<BN, FFB_EPI_BIAS_RES>(ta, tw, to, ba, grid, stream);
    case FFB_EPI_BIAS_GELU_TANH: return launch_instance<BN, FFB_EPI_BIAS_GELU_TANH>(ta, tw, to, ba, grid, stream);
    default: return launch_instance<BN, FFB_EPI_BIAS_GELU_ERF>(ta, tw, to, ba, grid, stream);
  }
}

// Plan of the smallest estimated time, in microseconds, from a model fitted to CUDA-graph
// timings of this kernel on the B200 (vision tower shapes, M = 256 .. 1024):
//   persistent, unsplit:   F + waves x K blocks x t_kb
//   cluster split S (256): F_S + K blocks / S x t_kb      (tiles x S <= SMs, one wave)
// with t_kb = 0.28 us per 64-element K block for 64 / 128-wide tiles and 0.32 for 256-wide
// ones (a CTA's single accumulator chain costs about the same per tcgen05.mma whatever its
// N, so a wide tile does more work per K block), F = 5.3 / 6.0 us of fixed cost, and the
// cluster reduction's F_2 = 6.5, F_4 = 8.6 us.  Measured: fc2 (1024 x 1024 x 4096) 23.1 us
// unsplit at 64 wide -> 14.2 us as 256-wide tiles split 4 ways; proj (K = 1024) 9.7 -> 9.0
// split 2 ways; qkv / fc1 stay unsplit 256-wide (10.8 / 20.2 us).  The plane split path
// (other widths or split counts) is slower everywhere and is never planned.
void auto_plan(int M, int N, int K, int& bn_out, int& splits_out) {
  const int sms = ffb::sm_count();
  const long long ttiles = (M + BM - 1) / BM, nkb = (K + BKE - 1) / BKE;
  double best = -1.0;
  bn_out = 256;
  splits_out = 1;
  for (int bn : {256, 128, 64}) {
    const long long tiles = ttiles * ((N + bn - 1) / bn);
    const long long waves = (tiles + sms - 1) / sms;
    const double t_kb = bn == 256 ? 0.32 : 0.28;
    const double cost = (bn == 256 ? 6.0 : 5.3) + (double)(waves * nkb) * t_kb;
    if (best < 0.0 || cost < best) {
      best = cost;
      bn_out = bn;
      splits_out = 1;
    }
  }
  const long long tiles256 = ttiles * ((N + 255) / 256);
  for (int sp : {2, 4}) {
    if (tiles256 * sp > sms || sp > nkb) continue;
    const double cost = (sp == 2 ? 6.5 : 8.6) + (double)((nkb + sp - 1) / sp) * 0.32;
    if (cost < best) {
      best = cost;
      bn_out = 256;
      splits_out = sp;
    }
  }
}

}  // namespace

extern "C" int ffb_bf16_gemm_plan(int M, int N, int K, int* plan) {
  FFB_REQUIRE(plan != nullptr, "ffb_bf16_gemm_plan: NULL plan");
  FFB_REQUIRE(M > 0 && N > 0 && K > 0, "ffb_bf16_gemm_plan: bad shape M=%d N=%d K=%d", M, N, K);
  auto_plan(M, N, K, plan[0], plan[1]);
  // counters the call needs: one per output tile for the plane split-K path, none otherwise
  plan[2] = plan[1] > 1 && !cluster_split(plan[0], plan[1]) ? ((M + BM - 1) / BM) * ((N + plan[0] - 1) / plan[0]) : 0;
  return FFB_OK;
}

extern "C" int ffb_bf16_gemm(const uint16_t* a, const uint16_t* w, const uint16_t* bias, const uint16_t* res,
                             int epilogue, uint16_t* out, int feature_tile, int splits, float* ws, uint32_t* counters,
                             int M, int N, int K, void* stream) {
  FFB_REQUIRE(a && w && out, "ffb_bf16_gemm: NULL operand");
  FFB_REQUIRE(M > 0 && N > 0 && K > 0, "ffb_bf16_gemm: bad shape M=%d N=%d K=%d", M, N, K);
  FFB_REQUIRE(K % 8 == 0 && N % 8 == 0, "ffb_bf16_gemm: K=%d and N=%d must be multiples of 8", K, N);
  FFB_REQUIRE(ffb::aligned(a, 16) && ffb::aligned(w, 16) && ffb::aligned(out, 16) &&
                  (!bias || ffb::aligned(bias, 16)) && (!res || ffb::aligned(res, 16)),
              "ffb_bf16_gemm: pointers must be 16-byte aligned");
  FFB_REQUIRE(epilogue == FFB_EPI_BIAS || epilogue == FFB_EPI_BIAS_RES || epilogue == FFB_EPI_BIAS_GELU_TANH ||
                  epilogue == FFB_EPI_BIAS_GELU_ERF,
              "ffb_bf16_gemm: unknown epilogue %d", epilogue);
  FFB_REQUIRE(epilogue != FFB_EPI_BIAS_RES || res != nullptr, "ffb_bf16_gemm: BIAS_RES needs res");
  const int nkb = (K + BKE - 1) / BKE;
  FFB_REQUIRE(splits >= 1 && splits <= 16 && splits <= nkb, "ffb_bf16_gemm: splits=%d outside [1, %d]", splits,
              nkb < 16 ? nkb : 16);
  int bn = feature_tile;
  if (bn <= 0) {
    int sp;
    auto_plan(M, N, K, bn, sp);
  }
  FFB_REQUIRE(bn == 64 || bn == 128 || bn == 256, "ffb_bf16_gemm: feature tile %d (64, 128 or 256)", bn);
  const bool cluster = cluster_split(bn, splits);
  FFB_REQUIRE(splits == 1 || cluster || (ws && counters && ffb::aligned(ws, 16) && ffb::aligned(counters, 4)),
              "ffb_bf16_gemm: splits > 1 (other than a 256-wide tile split 2 or 4 ways) needs ws (16-byte "
              "aligned) and counters");
  CUtensorMap ta, tw, to;
  int rc = ffb::make_tmap_2d(&ta, a, (uint64_t)M, (uint64_t)K, (uint64_t)K * 2, BM, BKE, 2);
  if (!rc) rc = ffb::make_tmap_2d(&tw, w, (uint64_t)N, (uint64_t)K, (uint64_t)K * 2, (uint32_t)bn, BKE, 2);
  if (!rc) rc = ffb::make_tmap_out(&to, out, 2, (uint64_t)N, (uint64_t)M, 1, (uint64_t)N * 2, (uint64_t)N * M * 2, 32, 32);
  if (rc) return rc;
  BArgs ba = {};
  ba.bias = bias;
  ba.res = res;
  ba.out = out;
  ba.ws = ws;
  ba.counters = counters;
  ba.splits = splits;
  ba.M = M;
  ba.N = N;
  ba.K = K;
  ba.n_ttiles = (M + BM - 1) / BM;
  ba.n_tiles = ba.n_ttiles * ((N + bn - 1) / bn) * splits;
  const int sms = ffb::sm_count();
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (cluster) {  // one CTA per (tile, split), clusters of `splits` CTAs
    cudaError_t e = splits == 2 ? launch_cluster_epi<2>(epilogue, ta, tw, ba, ba.n_tiles, s)
                                : launch_cluster_epi<4>(epilogue, ta, tw, ba, ba.n_tiles, s);
    if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_bf16_gemm: cluster launch: %s", cudaGetErrorString(e));
    return FFB_OK;
  }
  const int grid = ba.n_tiles < sms ? ba.n_tiles : sms;
  cudaError_t e = bn == 256 ? launch_epi<256>(epilogue, ta, tw, to, ba, grid, s)
                  : bn == 128 ? launch_epi<128>(epilogue, ta, tw, to, ba, grid, s)
                              : launch_epi<64>(epilogue, ta, tw, to, ba, grid, s);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_bf16_gemm: launch: %s", cudaGetErrorString(e));
  return FFB_OK;
}
