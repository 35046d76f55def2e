// W4A16 linear on the sm_100a tensor cores: bf16 activations x int4 weights (symmetric,
// group 128 along K, bf16 group scales), dequantised to bf16 in shared memory and
// multiplied with tcgen05.mma kind::f16 (bf16 x bf16 -> fp32 in tensor memory).
//
// Replaces the reference's `Int4.__call__` (_family/night_runtime.py:31-42, tinygemm
// `_weight_int4pack_mm`) for the W4A16 configuration.  Dequantisation follows the
// packing of ffb_pack_int4: nibble = q & 0xF (low nibble = even k), w = bf16(q * s).
//
// Tile = 128 tokens x BN output features, 64 K elements (one 128-byte bf16 swizzle row)
// per stage.  Persistent kernel, one CTA per SM, tiles round-robin (token tile fastest).
// Roles (576 threads):
//   warp 0       TMA producer: bf16 activation tile [128 x 64] (128-byte swizzle) and the
//                packed weight tile [BN rows x 32 bytes] into a ring of STAGES slots;
//   warp 1       TMEM allocator + single-thread MMA issuer (4 x K=16 MMAs per stage);
//   warps 2..9   converters: packed nibbles of slot s -> bf16 weight tile in one of two
//                swizzled buffers (the layout TMA would write), fence to the async proxy;
//                each thread owns a fixed row (half a row for BN = 128) and holds its group
//                scale and, fetched one group ahead, the next one, so the scale loads never
//                stall the conversion;
//   warps 10..17 epilogue, as in the FP8 GEMM (no scales: they are inside the weights).
// Barriers: full[s] (TMA), empty[s] (MMA done with the slot), wfull[j] (converters done),
// wempty[j] (MMA done with the bf16 tile), tfull/tempty (two TMEM accumulators).  Every
// wait is bounded; a timeout sets the abort flag and the device error word.
#include "common.cuh"
#include "pdl.cuh"

#include <string.h>

namespace {

constexpr int BM = 128;                 // tokens per tile (UMMA M)
constexpr int BKE = 64;                 // K elements per stage
constexpr int UMMA_K = 16;              // K per tcgen05.mma for 16-bit operands
constexpr int A_BYTES = BM * BKE * 2;   // 16 KB
constexpr int CONV_WARPS = 8;
constexpr int NWB = 2;  // bf16 weight buffers (three measured no faster and cost a TMA stage)
constexpr int EPI_WARPS = 8;
constexpr int EPI_WARP0 = 2 + CONV_WARPS;
constexpr int THREADS = 64 + (CONV_WARPS + EPI_WARPS) * 32;
constexpr int SMEM_LIMIT = 232448;

template <int BN>
struct W4Cfg {
  static constexpr int WP_BYTES = BN * BKE / 2;      // packed nibbles, 32 bytes per row
  static constexpr int STAGE_BYTES = A_BYTES + WP_BYTES;
  static constexpr int WB_BYTES = BN * BKE * 2;      // bf16 weight tile, 128-byte rows
  static constexpr int STG_BYTES = EPI_WARPS * 2 * 2048;
  static constexpr int FIXED = NWB * WB_BYTES + STG_BYTES + 512 + 1024;
  static constexpr int FIT = (SMEM_LIMIT - FIXED) / STAGE_BYTES;
  static constexpr int STAGES = FIT > 8 ? 8 : FIT;
  static constexpr int SMEM = STAGES * STAGE_BYTES + FIXED;
  static constexpr int TMEM_COLS = 2 * BN;
  static_assert(BN == 128 || BN == 256, "feature tile must be 128 or 256");
  static_assert(STAGE_BYTES % 1024 == 0 && WB_BYTES % 1024 == 0, "swizzled tiles need 1024-byte alignment");
};

struct W4Args {
  const uint16_t* scales;  // [N][K/128] bf16
  int M, N, K, n_ttiles, splits, n_tiles;
};

__device__ __forceinline__ void tile_coords(const W4Args& a, int t, int& tt, int& ks, int& ft) {
  tt = t % a.n_ttiles;
  const int rest = t / a.n_ttiles;
  ks = rest % a.splits;
  ft = rest / a.splits;
}
__device__ __forceinline__ void k_range(const W4Args& a, int ks, int nkb, int& kb0, int& kb1) {
  kb0 = (int)((long long)ks * nkb / a.splits);
  kb1 = (int)((long long)(ks + 1) * nkb / a.splits);
}
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}

// Eight nibbles (k = 8c .. 8c+7, low nibble first) -> four bf16x2 words of q * s.
// bf16(128 + u) has the bits 0x4300 | u for u < 128, so with u = nibble ^ 8 the value
// minus 136 is q exactly; the bf16 multiply by s then rounds q * s to nearest even.
__device__ __forceinline__ uint4 dequant8(uint32_t nib8, __nv_bfloat162 s2) {
  const uint32_t u = nib8 ^ 0x88888888u;
  const __nv_bfloat162 off = __float2bfloat162_rn(136.f);
  uint32_t w[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const uint32_t lo = (u >> (8 * p)) & 0xFu, hi = (u >> (8 * p + 4)) & 0xFu;
    const uint32_t bits = 0x43004300u | lo | (hi << 16);
    __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162*>(&bits);
    x = __hsub2(x, off);   // exact: small integers
    x = __hmul2(x, s2);    // round to nearest even
    w[p] = *reinterpret_cast<const uint32_t*>(&x);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    w4a16_gemm_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_w,
                      const __grid_constant__ CUtensorMap tmap_o, const W4Args args) {
  using C = W4Cfg<BN>;
  static_assert(EPI != FFB_EPI_SWIGLU || BN == 256, "gate/up pairs of 128 channels per tile");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* wb_all = smem + C::STAGES * C::STAGE_BYTES;  // [NWB][WB_BYTES], 1024-aligned
  uint8_t* stg_all = wb_all + NWB * C::WB_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(stg_all + C::STG_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* wfull = empty + C::STAGES;  // [NWB]
  uint64_t* wempty = wfull + NWB;       // [NWB]
  uint64_t* tfull = wempty + NWB;       // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nkb = args.K / BKE;

  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NWB; ++b) {
      mbar_init(&wfull[b], CONV_WARPS);
      mbar_init(&wempty[b], 1);
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
      int pre = 0;
      if ((int)blockIdx.x < args.n_tiles) {  // weights do not depend on the previous kernel
        int tt, ks, ft, kb0, kb1;
        tile_coords(args, blockIdx.x, tt, ks, ft);
        k_range(args, ks, nkb, kb0, kb1);
        pre = kb1 - kb0 < C::STAGES ? kb1 - kb0 : C::STAGES;
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
          tma_load_2d(smem + i * C::STAGE_BYTES + A_BYTES, &tmap_w, &full[i], (kb0 + i) * (BKE / 2), ft * BN, pol_w);
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
          if (it < pre) {
            tma_load_2d(st, &tmap_a, &full[s], kb * BKE, tt * BM, pol_a);
            continue;
          }
          if (!mbar_wait_bounded(&empty[s], ((uint32_t)(it / C::STAGES) & 1u) ^ 1u, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_2d(st, &tmap_a, &full[s], kb * BKE, tt * BM, pol_a);
          tma_load_2d(st + A_BYTES, &tmap_w, &full[s], kb * (BKE / 2), ft * BN, pol_w);
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
      constexpr uint32_t idesc = idesc_bf16(BM, BN);
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
          const int s = it % C::STAGES, j = it % NWB;
          if (!mbar_wait_bounded(&full[s], (uint32_t)(it / C::STAGES) & 1u, abort_flag) ||
              !mbar_wait_bounded(&wfull[j], (uint32_t)(it / NWB) & 1u, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(smem_u32(smem + s * C::STAGE_BYTES));
          const uint64_t dw = umma_desc_sw128(smem_u32(wb_all + j * C::WB_BYTES));
#pragma unroll
          for (int kk = 0; kk < BKE / UMMA_K; ++kk)  // +32 bytes per K step = +2 encoded
            umma_f16(acc, da + 2 * kk, dw + 2 * kk, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
          umma_commit(&wempty[j]);
        }
        umma_commit(&tfull[buf]);
        if (!ok) {
          *abort_flag = 1;
          break;
        }
      }
    }
  } else if (warp < EPI_WARP0) {
    // ------------------------------------------------------------------ converters
    pdl_wait();
    constexpr int CT = CONV_WARPS * 32;
    constexpr int CPT = BN * 8 / CT;  // 16-byte output chunks per thread and stage (8 or 4)
    static_assert(CPT == 8 || CPT == 4, "a whole or half 64-element row per converter thread");
    const int ct = tid - 64;
    const int row = ct * CPT / 8, c0 = ct * CPT % 8;
    const int groups = args.K / 128;
    int it = 0;
    for (int t = blockIdx.x; t < args.n_tiles && !*abort_flag; t += gridDim.x) {
      int tt, ks, ft, kb0, kb1;
      tile_coords(args, t, tt, ks, ft);
      k_range(args, ks, nkb, kb0, kb1);
      // this row's scale of the current 128-element group and of the next one (the load is
      // issued a whole group, two stages, before its first use)
      const uint16_t* srow = args.scales + (size_t)(ft * BN + row) * groups;
      int g = kb0 >> 1;
      uint16_t s_cur = srow[g];
      uint16_t s_nxt = g + 1 < groups ? srow[g + 1] : (uint16_t)0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb, ++it) {
        const int s = it % C::STAGES, j = it % NWB;
        if ((kb >> 1) != g) {
          g = kb >> 1;
          s_cur = s_nxt;
          s_nxt = g + 1 < groups ? srow[g + 1] : (uint16_t)0;
        }
        if (!mbar_wait_bounded(&full[s], (uint32_t)(it / C::STAGES) & 1u, abort_flag) ||
            !mbar_wait_bounded(&wempty[j], ((uint32_t)(it / NWB) & 1u) ^ 1u, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t* wp = smem + s * C::STAGE_BYTES + A_BYTES + row * 32 + c0 * 4;
        uint32_t nib[CPT];
        const uint4 p0 = *reinterpret_cast<const uint4*>(wp);
        nib[0] = p0.x;
        nib[1] = p0.y;
        nib[2] = p0.z;
        nib[3] = p0.w;
        if constexpr (CPT == 8) {
          const uint4 p1 = *reinterpret_cast<const uint4*>(wp + 16);
          nib[4] = p1.x;
          nib[5] = p1.y;
          nib[6] = p1.z;
          nib[7] = p1.w;
        }
        const __nv_bfloat162 s2 = __halves2bfloat162(__ushort_as_bfloat16(s_cur), __ushort_as_bfloat16(s_cur));
        uint8_t* dst = wb_all + j * C::WB_BYTES + row * 128;
#pragma unroll
        for (int c = 0; c < CPT; ++c)  // 16-byte chunk c0 + c of the row, 128-byte swizzle
          *reinterpret_cast<uint4*>(dst + (((c0 + c) ^ (row & 7)) << 4)) = dequant8(nib[c], s2);
        fence_proxy_async_smem();  // the bf16 tile is read by the tensor core (async proxy)
        __syncwarp();
        if (lane == 0) mbar_arrive(&wfull[j]);
      }
      if (!ok) {
        *abort_flag = 1;
        break;
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue
    pdl_wait();
    if (warp == EPI_WARP0 && lane == 0) pdl_launch();
    const int q = warp & 3;                    // TMEM lane quarter = this warp's 32 tokens
    const int half = (warp - EPI_WARP0) >> 2;  // which half of the tile's columns
    int lt = 0;
    uint32_t sc = 0;
    for (int t = blockIdx.x; t < args.n_tiles; t += gridDim.x, ++lt) {
      int tt, ks, ft;
      tile_coords(args, t, tt, ks, ft);
      const int buf = lt & 1;
      if (!(mbar_wait_bounded(&tfull[buf], (uint32_t)(lt >> 1) & 1u, abort_flag) && !*abort_flag)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t acc = tmem + (uint32_t)(buf * BN) + ((uint32_t)(q * 32) << 16);
      const int n0 = ft * BN;
      auto staged_store = [&](const uint32_t (&w16)[16], int x, int z) {
        uint8_t* sb = stg_all + ((warp - EPI_WARP0) * 2 + (sc & 1)) * 2048;
        if (lane == 0) bulk_wait_read<1>();
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
      if constexpr (EPI == FFB_EPI_SWIGLU) {
        constexpr int HALFC = BN / 2;
        const int cb = half * (HALFC / 2);
#pragma unroll 1
        for (int c0 = cb; c0 < cb + HALFC / 2; c0 += 32) {
          uint32_t o[16];
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
#pragma unroll
            for (int j = 0; j < 8; j += 2) {
              float y2[2];
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const float gv = round_bf(__uint_as_float(g[cur][j + h]));  // bf16 gate
                const float uv = round_bf(__uint_as_float(u[cur][j + h]));  // bf16 up
                y2[h] = silu_lookup(gv) * uv;
              }
              o[grp * 4 + (j >> 1)] = pack2(y2[0], y2[1]);
            }
            if (grp < 3) {
              tmem_wait_ld();
              reg_fence(g[cur ^ 1]);
              reg_fence(u[cur ^ 1]);
            }
          }
          staged_store(o, ft * HALFC + c0, 0);
        }
      } else if constexpr (EPI == FFB_EPI_F32_PARTIAL) {
#pragma unroll 1
        for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 16) {
          uint32_t r[16];
          tmem_ld16_async(acc + (uint32_t)c, r);
          tmem_wait_ld();
          reg_fence(r);
          staged_store(r, n0 + c, ks);
        }
      } else {
#pragma unroll 1
        for (int c = half * (BN / 2); c < (half + 1) * (BN / 2); c += 32) {
          uint32_t r0[16], r1[16];
          tmem_ld16_async(acc + (uint32_t)c, r0);
          tmem_ld16_async(acc + (uint32_t)(c + 16), r1);
          tmem_wait_ld();
          reg_fence(r0);
          reg_fence(r1);
          uint32_t o[16];
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            o[j >> 1] = pack2(__uint_as_float(r0[j]), __uint_as_float(r0[j + 1]));
            o[8 + (j >> 1)] = pack2(__uint_as_float(r1[j]), __uint_as_float(r1[j + 1]));
          }
          staged_store(o, n0 + c, 0);
        }
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
  if (tid == 0 && *abort_flag) atomicOr(&ffb_device_error_word, ffb::ERR_W4_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

int num_sms() { return ffb::sm_count(); }

template <int BN, int EPI>
cudaError_t launch_instance(const CUtensorMap& ta, const CUtensorMap& tw, const CUtensorMap& to, const W4Args& wa,
                            int grid, cudaStream_t stream) {
  using C = W4Cfg<BN>;
  cudaError_t e = ffb::set_smem_attr(reinterpret_cast<const void*>(w4a16_gemm_kernel<BN, EPI>), C::SMEM);
  if (e != cudaSuccess) return e;
  return ffb::launch(w4a16_gemm_kernel<BN, EPI>, dim3(grid), dim3(THREADS), C::SMEM, stream, ta, tw, to, wa);
}

template <int BN>
int launch_bn(const uint16_t* x, const uint8_t* packed, int epilogue, uint16_t* out, float* ws, W4Args& wa,
              cudaStream_t stream) {
  CUtensorMap ta, tw, to;
  int rc = ffb::make_tmap_2d(&ta, x, (uint64_t)wa.M, (uint64_t)wa.K, (uint64_t)wa.K * 2, BM, BKE, 2);
  if (!rc) rc = ffb::make_tmap_2d_bytes(&tw, packed, (uint64_t)wa.N, (uint64_t)wa.K / 2, (uint64_t)wa.K / 2, BN,
                                        BKE / 2);
  if (!rc && epilogue == FFB_EPI_BF16)
    rc = ffb::make_tmap_out(&to, out, 2, wa.N, wa.M, 1, (uint64_t)wa.N * 2, (uint64_t)wa.N * wa.M * 2, 32, 32);
  if (!rc && epilogue == FFB_EPI_SWIGLU)
    rc = ffb::make_tmap_out(&to, out, 2, wa.N / 2, wa.M, 1, (uint64_t)wa.N, (uint64_t)wa.N * wa.M, 32, 32);
  if (!rc && epilogue == FFB_EPI_F32_PARTIAL)
    rc = ffb::make_tmap_out(&to, ws, 4, wa.N, wa.M, wa.splits, (uint64_t)wa.N * 4, (uint64_t)wa.N * wa.M * 4, 16, 32);
  if (rc) return rc;
  wa.n_ttiles = (wa.M + BM - 1) / BM;
  wa.n_tiles = (wa.N / BN) * wa.splits * wa.n_ttiles;
  const int grid = wa.n_tiles < num_sms() ? wa.n_tiles : num_sms();
  if (epilogue == FFB_EPI_SWIGLU) {
    rc = ffb::ensure_silu_table(stream);
    if (rc) return rc;
  }
  cudaError_t e = cudaErrorInvalidValue;
  if constexpr (BN == 256) {
    if (epilogue == FFB_EPI_SWIGLU) e = launch_instance<256, FFB_EPI_SWIGLU>(ta, tw, to, wa, grid, stream);
    else if (epilogue == FFB_EPI_BF16) e = launch_instance<256, FFB_EPI_BF16>(ta, tw, to, wa, grid, stream);
    else e = launch_instance<256, FFB_EPI_F32_PARTIAL>(ta, tw, to, wa, grid, stream);
  } else {
    if (epilogue == FFB_EPI_BF16) e = launch_instance<128, FFB_EPI_BF16>(ta, tw, to, wa, grid, stream);
    else e = launch_instance<128, FFB_EPI_F32_PARTIAL>(ta, tw, to, wa, grid, stream);
  }
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_w4a16_gemm: launch: %s", cudaGetErrorString(e));
  return FFB_OK;
}

}  // namespace

extern "C" int ffb_w4a16_gemm(const uint16_t* x, const uint8_t* packed, const uint16_t* scales, int epilogue,
                              uint16_t* out, float* ws, int splits, int feature_tile, int M, int N, int K,
                              void* stream) {
  FFB_REQUIRE(x && packed && scales, "ffb_w4a16_gemm: NULL operand");
  FFB_REQUIRE(M > 0 && N > 0 && K > 0, "ffb_w4a16_gemm: bad shape M=%d N=%d K=%d", M, N, K);
  FFB_REQUIRE(K % 128 == 0, "ffb_w4a16_gemm: K=%d must be a multiple of the group size 128", K);
  FFB_REQUIRE(N % 128 == 0, "ffb_w4a16_gemm: N=%d must be a multiple of 128", N);
  FFB_REQUIRE(ffb::aligned(x, 16) && ffb::aligned(packed, 16), "ffb_w4a16_gemm: operands must be 16-byte aligned");
  FFB_REQUIRE(epilogue == FFB_EPI_BF16 || epilogue == FFB_EPI_F32_PARTIAL || epilogue == FFB_EPI_SWIGLU,
              "ffb_w4a16_gemm: unknown epilogue %d", epilogue);
  const int nkb = K / BKE;
  if (epilogue == FFB_EPI_F32_PARTIAL) {
    FFB_REQUIRE(ws != nullptr && ffb::aligned(ws, 16), "ffb_w4a16_gemm: F32_PARTIAL needs a 16-byte aligned ws");
    FFB_REQUIRE(splits >= 1 && splits <= nkb, "ffb_w4a16_gemm: splits=%d outside [1, %d]", splits, nkb);
  } else {
    FFB_REQUIRE(out != nullptr && ffb::aligned(out, 16), "ffb_w4a16_gemm: out must be non-NULL, 16-byte aligned");
    FFB_REQUIRE(splits == 1, "ffb_w4a16_gemm: splits must be 1 unless the epilogue is F32_PARTIAL");
  }
  int bn = feature_tile > 0 ? feature_tile : (N % 256 == 0 ? 256 : 128);
  if (epilogue == FFB_EPI_SWIGLU) bn = 256;
  FFB_REQUIRE(bn == 128 || bn == 256, "ffb_w4a16_gemm: feature tile %d (128 or 256)", bn);
  FFB_REQUIRE(N % bn == 0, "ffb_w4a16_gemm: N=%d must be a multiple of the feature tile %d", N, bn);
  W4Args wa = {};
  wa.scales = scales;
  wa.M = M;
  wa.N = N;
  wa.K = K;
  wa.splits = splits;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return bn == 256 ? launch_bn<256>(x, packed, epilogue, out, ws, wa, s)
                   : launch_bn<128>(x, packed, epilogue, out, ws, wa, s);
}
