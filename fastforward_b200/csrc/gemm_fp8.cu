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
//   warps 2..9  epilogue: warp w reads TMEM lanes 32*(w%4).. (its 32 tokens) and half of
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
constexpr int EPI_WARPS = 8;
constexpr int THREADS = 64 + EPI_WARPS * 32;
constexpr int SMEM_LIMIT = 232448;
constexpr int EPI_QKROPE = 100;  // internal epilogue code of ffb_fp8_gemm_qk_rope

template <int BN>
struct Cfg {
  static constexpr int B_TILE_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = A_TILE_BYTES + B_TILE_BYTES;
  static constexpr int STG_BYTES = EPI_WARPS * 2 * 2048;  // per warp: 2 x [32 rows x 64 B] store staging
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

struct GemmArgs {
  const float* a_scale;
  const float* w_scale;
  uint16_t* out;
  float* ws;
  int a_per_row, w_per_col, epilogue;
  int M, N, K, n_ttiles, splits, n_tiles;
  RopeSide rope;
};

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
__device__ __forceinline__ float wsc(const GemmArgs& a, int n) { return a.w_per_col ? a.w_scale[n] : a.w_scale[0]; }

// Per-head RMSNorm + rotate-half RoPE of one token's 128-wide head held as packed bf16
// pairs x[64] (elements 2i, 2i+1 in the low/high halves of x[i]); writes the 128 outputs
// to dst.  Rounding as _legacy/lower_kernels.py:66-86, statistics as inv_rms_from_ss.
__device__ __forceinline__ void qk_rope_row(const uint32_t (&x)[64], const uint16_t* __restrict__ wn,
                                            const uint16_t* __restrict__ cosr, const uint16_t* __restrict__ sinr,
                                            float eps, uint16_t* __restrict__ dst) {
  double ss = 0.0;
#pragma unroll
  for (int i = 0; i < 64; ++i) {
    const float a = lo_bf(x[i]), b = hi_bf(x[i]);
    ss += (double)(a * a) + (double)(b * b);
  }
  const float inv = inv_rms_from_ss(ss, 128, eps);
  // elements e and e+64 are rotate-half partners: handle 8 of each per step
#pragma unroll
  for (int e0 = 0; e0 < 64; e0 += 8) {
    const uint4 w0 = *reinterpret_cast<const uint4*>(wn + e0);
    const uint4 w1 = *reinterpret_cast<const uint4*>(wn + e0 + 64);
    const uint4 c0 = *reinterpret_cast<const uint4*>(cosr + e0);
    const uint4 c1 = *reinterpret_cast<const uint4*>(cosr + e0 + 64);
    const uint4 s0 = *reinterpret_cast<const uint4*>(sinr + e0);
    const uint4 s1 = *reinterpret_cast<const uint4*>(sinr + e0 + 64);
    const uint32_t wa[4] = {w0.x, w0.y, w0.z, w0.w}, wb[4] = {w1.x, w1.y, w1.z, w1.w};
    const uint32_t ca[4] = {c0.x, c0.y, c0.z, c0.w}, cb[4] = {c1.x, c1.y, c1.z, c1.w};
    const uint32_t sa[4] = {s0.x, s0.y, s0.z, s0.w}, sb[4] = {s1.x, s1.y, s1.z, s1.w};
    uint32_t ya[4], yb[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int i = (e0 >> 1) + p;  // packed index of elements e0+2p, e0+2p+1
      const uint32_t xa = x[i], xb = x[i + 32];
      float out_a[2], out_b[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float va = h ? hi_bf(xa) : lo_bf(xa);  // element e (< 64)
        const float vb = h ? hi_bf(xb) : lo_bf(xb);  // element e + 64
        const float na = round_bf(round_bf(va * inv) * (h ? hi_bf(wa[p]) : lo_bf(wa[p])));
        const float nb = round_bf(round_bf(vb * inv) * (h ? hi_bf(wb[p]) : lo_bf(wb[p])));
        const float cea = h ? hi_bf(ca[p]) : lo_bf(ca[p]), ceb = h ? hi_bf(cb[p]) : lo_bf(cb[p]);
        const float sea = h ? hi_bf(sa[p]) : lo_bf(sa[p]), seb = h ? hi_bf(sb[p]) : lo_bf(sb[p]);
        out_a[h] = round_bf(na * cea) + round_bf(-nb * sea);  // y[e]    = xn[e]*c - xn[e+64]*s
        out_b[h] = round_bf(nb * ceb) + round_bf(na * seb);   // y[e+64] = xn[e+64]*c + xn[e]*s
      }
      ya[p] = pack2(out_a[0], out_a[1]);
      yb[p] = pack2(out_b[0], out_b[1]);
    }
    *reinterpret_cast<uint4*>(dst + e0) = make_uint4(ya[0], ya[1], ya[2], ya[3]);
    *reinterpret_cast<uint4*>(dst + e0 + 64) = make_uint4(yb[0], yb[1], yb[2], yb[3]);
  }
}

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ CUtensorMap tmap_o, const GemmArgs args) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stg_all = smem + C::STAGES * C::STAGE_BYTES;  // 1024-aligned
  uint64_t* full = reinterpret_cast<uint64_t*>(stg_all + C::STG_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;  // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_a);
    tma_prefetch_desc(&tmap_w);
    if (args.epilogue != EPI_QKROPE) tma_prefetch_desc(&tmap_o);
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
      int pre = 0;
      if ((int)blockIdx.x < args.n_tiles) {
        int tt, ks, ft, kb0, kb1;
        tile_coords(args, blockIdx.x, tt, ks, ft);
        k_range(args, ks, nkb, kb0, kb1);
        pre = kb1 - kb0 < C::STAGES ? kb1 - kb0 : C::STAGES;
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
          tma_load_2d(smem + i * C::STAGE_BYTES + A_TILE_BYTES, &tmap_w, &full[i], (kb0 + i) * BK, ft * BN, pol_w);
        }
      }
      pdl_wait();
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
    const int half = (warp - 2) >> 2;  // which half of the tile's columns
    int lt = 0;
    uint32_t sc = 0;                   // staged-store counter (selects the staging buffer)
    for (int t = blockIdx.x; t < args.n_tiles; t += gridDim.x, ++lt) {
      int tt, ks, ft;
      tile_coords(args, t, tt, ks, ft);
      const int buf = lt & 1;
      // each epilogue warp waits on its own; a timeout makes every one of them stop
      if (!(mbar_wait_bounded(&tfull[buf], (uint32_t)(lt >> 1) & 1u, abort_flag) && !*abort_flag)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int m = tt * BM + q * 32 + lane;  // this thread's token
      const bool row_ok = m < args.M;
      const float sa = args.a_per_row ? (row_ok ? args.a_scale[m] : 0.f) : args.a_scale[0];
      const uint32_t acc = tmem + (uint32_t)(buf * BN) + ((uint32_t)(q * 32) << 16);
      const int n0 = ft * BN;

      if (args.epilogue == EPI_QKROPE) {
        // one head per tile (BN == 128); the first four warps own the whole row
        if (half == 0) {
          uint32_t x[64];
#pragma unroll
          for (int c = 0; c < 128; c += 16) {
            float v[16];
            tmem_ld16(acc + (uint32_t)c, v);
#pragma unroll
            for (int j = 0; j < 16; j += 2)  // the linear's bf16 output
              x[(c + j) >> 1] = pack2(v[j] * sa * wsc(args, n0 + c + j), v[j + 1] * sa * wsc(args, n0 + c + j + 1));
          }
          if (row_ok) {
            const RopeSide& r = args.rope;
            const size_t T = (size_t)args.M;
            if (ft < r.HQ + r.HK) {
              const bool is_q = ft < r.HQ;
              uint16_t* dst = is_q ? r.yq + ((size_t)ft * T + m) * 128 : r.yk + ((size_t)(ft - r.HQ) * T + m) * 128;
              qk_rope_row(x, is_q ? r.q_norm : r.k_norm, r.cos + (size_t)m * 128, r.sin + (size_t)m * 128, r.eps,
                          dst);
            } else {
              uint16_t* dst = r.yv + ((size_t)(ft - r.HQ - r.HK) * T + m) * 128;
#pragma unroll
              for (int i = 0; i < 64; i += 4)
                *reinterpret_cast<uint4*>(dst + 2 * i) = make_uint4(x[i], x[i + 1], x[i + 2], x[i + 3]);
            }
          }
        }
      } else {
        // Staged stores: the warp writes its [32 tokens x 64 B] chunk into one of its two
        // swizzled staging buffers and lane 0 issues a TMA store (rows >= M are clipped).
        auto staged_store = [&](const uint32_t (&w16)[16], int x, int z) {
          uint8_t* sb = stg_all + ((warp - 2) * 2 + (sc & 1)) * 2048;
          if (lane == 0) bulk_wait_read<1>();  // the store that used this buffer has read it
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
        if (args.epilogue == FFB_EPI_SWIGLU) {
          // columns [0, BN/2) are gate channels ft*BN/2 + j, [BN/2, BN) the matching up rows
          constexpr int HALFC = BN / 2;
#pragma unroll 1
          for (int c = half * (HALFC / 2); c < (half + 1) * (HALFC / 2); c += 32) {
            uint32_t o[16];
#pragma unroll
            for (int sub = 0; sub < 32; sub += 16) {
              float g[16], u[16];
              tmem_ld16(acc + (uint32_t)(c + sub), g);
              tmem_ld16(acc + (uint32_t)(HALFC + c + sub), u);
#pragma unroll
              for (int j = 0; j < 16; j += 2) {
                float y2[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                  const int jj = sub + j + h;
                  const float gv = round_bf(g[j + h] * sa * wsc(args, n0 + c + jj));          // bf16 gate
                  const float uv = round_bf(u[j + h] * sa * wsc(args, n0 + HALFC + c + jj));  // bf16 up
                  y2[h] = round_bf(__fdiv_rn(gv, 1.f + expf(-gv))) * uv;
                }
                o[(sub + j) >> 1] = pack2(y2[0], y2[1]);
              }
            }
            staged_store(o, ft * HALFC + c, 0);
          }
        } else if (args.epilogue == FFB_EPI_F32_PARTIAL) {
#pragma unroll 1
          for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 16) {
            float v[16];
            tmem_ld16(acc + (uint32_t)c, v);
            uint32_t o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = __float_as_uint(v[j] * sa * wsc(args, n0 + c + j));
            staged_store(o, n0 + c, ks);
          }
        } else {
#pragma unroll 1
          for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 32) {
            float v[32];
            tmem_ld32(acc + (uint32_t)c, v);
            uint32_t o[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2)
              o[j >> 1] = pack2(v[j] * sa * wsc(args, n0 + c + j), v[j + 1] * sa * wsc(args, n0 + c + j + 1));
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

int num_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) sms = 148;
  }
  return sms;
}

template <int BN>
int launch_bn(const uint8_t* a8, const uint8_t* w8, GemmArgs& ga, cudaStream_t stream) {
  using C = Cfg<BN>;
  CUtensorMap ta, tw, to;
  memset(&to, 0, sizeof(to));
  int rc = ffb::make_tmap_2d(&ta, a8, (uint64_t)ga.M, (uint64_t)ga.K, (uint64_t)ga.K, BM, BK, 1);
  if (!rc) rc = ffb::make_tmap_2d(&tw, w8, (uint64_t)ga.N, (uint64_t)ga.K, (uint64_t)ga.K, BN, BK, 1);
  if (!rc && ga.epilogue == FFB_EPI_BF16)
    rc = ffb::make_tmap_out(&to, ga.out, 2, ga.N, ga.M, 1, (uint64_t)ga.N * 2, (uint64_t)ga.N * ga.M * 2, 32, 32);
  if (!rc && ga.epilogue == FFB_EPI_SWIGLU)
    rc = ffb::make_tmap_out(&to, ga.out, 2, ga.N / 2, ga.M, 1, (uint64_t)ga.N, (uint64_t)ga.N * ga.M, 32, 32);
  if (!rc && ga.epilogue == FFB_EPI_F32_PARTIAL)
    rc = ffb::make_tmap_out(&to, ga.ws, 4, ga.N, ga.M, ga.splits, (uint64_t)ga.N * 4, (uint64_t)ga.N * ga.M * 4, 16,
                            32);
  if (rc) return rc;
  static bool attr_set = false;  // the attribute is per function (one device per process here)
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(fp8_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_fp8_gemm: smem attribute: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  ga.n_ttiles = (ga.M + BM - 1) / BM;
  ga.n_tiles = (ga.N / BN) * ga.splits * ga.n_ttiles;
  const int grid = ga.n_tiles < num_sms() ? ga.n_tiles : num_sms();
  cudaError_t e = ffb::launch(fp8_gemm_kernel<BN>, dim3(grid), dim3(THREADS), C::SMEM, stream, ta, tw, to, ga);
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
  return FFB_OK;
}

}  // namespace

extern "C" int ffb_fp8_gemm(const uint8_t* a8, const float* a_scale, int a_per_row, const uint8_t* w8,
                            const float* w_scale, int w_per_col, int epilogue, uint16_t* out, float* ws, int splits,
                            int feature_tile, int M, int N, int K, void* stream) {
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
  int bn = feature_tile > 0 ? feature_tile : (N % 256 == 0 ? 256 : 128);
  if (epilogue == FFB_EPI_SWIGLU) bn = 256;  // the gate/up interleave is per 128 channels
  FFB_REQUIRE(bn == 128 || bn == 256, "ffb_fp8_gemm: feature tile %d (128 or 256)", bn);
  FFB_REQUIRE(N % bn == 0, "ffb_fp8_gemm: N=%d must be a multiple of the feature tile %d", N, bn);
  GemmArgs ga = {};
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
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return bn == 256 ? launch_bn<256>(a8, w8, ga, s) : launch_bn<128>(a8, w8, ga, s);
}

extern "C" int ffb_fp8_gemm_qk_rope(const uint8_t* a8, const float* a_scale, int a_per_row, const uint8_t* w8,
                                    const float* w_scale, int w_per_col, const uint16_t* q_norm,
                                    const uint16_t* k_norm, float eps, const uint16_t* cos, const uint16_t* sin,
                                    uint16_t* yq, uint16_t* yk, uint16_t* yv, int T, int HQ, int HK, int K,
                                    void* stream) {
  const int N = (HQ + 2 * HK) * 128;
  int rc = check_common(a8, a_scale, w8, w_scale, T, N, K);
  if (rc) return rc;
  FFB_REQUIRE(q_norm && k_norm && cos && sin && yq && yk && yv, "ffb_fp8_gemm_qk_rope: NULL pointer");
  FFB_REQUIRE(HQ > 0 && HK > 0 && HQ % HK == 0, "ffb_fp8_gemm_qk_rope: bad heads HQ=%d HK=%d", HQ, HK);
  FFB_REQUIRE(ffb::aligned(q_norm, 16) && ffb::aligned(k_norm, 16) && ffb::aligned(cos, 16) && ffb::aligned(sin, 16) &&
                  ffb::aligned(yq, 16) && ffb::aligned(yk, 16) && ffb::aligned(yv, 16),
              "ffb_fp8_gemm_qk_rope: 16-byte alignment");
  GemmArgs ga = {};
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
  return launch_bn<128>(a8, w8, ga, reinterpret_cast<cudaStream_t>(stream));
}
