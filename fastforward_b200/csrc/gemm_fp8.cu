// FP8 e4m3 W8A8 linear on the sm_100a tensor cores (tcgen05, kind::f8f6f4).
//
// Replaces the reference's quantiser + torch._scaled_mm pair
// (_family/depth_fp8.py:22-26, _legacy/fp8_private.py:29-38).
//
// Orientation ("swap AB"): the weight tile is the 128-row UMMA A operand and the tokens
// are the UMMA N dimension, so a CTA owns 128 output features x BN tokens, its weight
// rows stream from HBM exactly once per token tile, and a prefill of T <= 256 tokens
// reads every weight byte once.  D[feature, token] accumulates in tensor memory (fp32).
//
// Roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + single-thread
// MMA issuer, warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31).
// Pipeline: STAGES smem slots, full[s] (TMA bytes landed) / empty[s] (MMAs that read
// the slot completed, signalled by tcgen05.commit); accum (all MMAs done).
// Every wait is bounded (mbar_wait_bounded); a timeout sets the CTA abort flag and the
// device error word, lets in-flight copies and MMAs drain, frees TMEM and returns.
#include "common.cuh"
#include "pdl.cuh"

namespace {

constexpr int BM = 128;        // features per CTA (UMMA M)
constexpr int BK = 128;        // K bytes per stage (one 128-byte swizzle atom row)
constexpr int UMMA_K = 32;     // K per tcgen05.mma for 8-bit operands
constexpr int W_TILE_BYTES = BM * BK;
constexpr int EPI_THREADS = 128;

__host__ __device__ constexpr int tmem_cols_for(int bn) {
  return bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : 256;
}
__host__ __device__ constexpr int stages_for(int bn) {
  return bn >= 224 ? 4 : bn >= 160 ? 5 : bn >= 96 ? 6 : 8;
}
template <int BN>
struct Cfg {
  static constexpr int A_TILE_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = W_TILE_BYTES + A_TILE_BYTES;
  static constexpr int STAGES = stages_for(BN);
  static constexpr int XCHG_BYTES = 64 * 16 * 4;  // SwiGLU gate/up exchange (64 rows x 16 cols fp32)
  static constexpr int SMEM = STAGES * STAGE_BYTES + XCHG_BYTES + 256 + 1024;  // + barriers + align slack
  static constexpr int TMEM_COLS = tmem_cols_for(BN);
};

struct GemmArgs {
  const float* a_scale;
  const float* w_scale;
  uint16_t* out;
  float* ws;
  int a_per_row, w_per_col, epilogue;
  int M, N, K, n_ttiles, splits;
};

template <int BN>
__global__ void __launch_bounds__(192, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                    const GemmArgs args) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES + C::XCHG_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* accum = empty + C::STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* xchg = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bid = blockIdx.x;
  const int tt = bid % args.n_ttiles;
  const int rest = bid / args.n_ttiles;
  const int ks = rest % args.splits;
  const int ft = rest / args.splits;
  const int n0 = ft * BM, m0 = tt * BN;
  const int nkb_total = (args.K + BK - 1) / BK;
  const int kb0 = (int)((long long)ks * nkb_total / args.splits);
  const int kb1 = (int)((long long)(ks + 1) * nkb_total / args.splits);
  const int nkb = kb1 - kb0;

  if (tid == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accum, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_w);
    tma_prefetch_desc(&tmap_a);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first(), pol_a = policy_evict_last();
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
        if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* st = smem + s * C::STAGE_BYTES;
        mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
        const int kx = (kb0 + i) * BK;
        tma_load_2d(st, &tmap_w, &full[s], kx, n0, pol_w);
        tma_load_2d(st + W_TILE_BYTES, &tmap_a, &full[s], kx, m0, pol_a);
        ++issued;
      }
      if (*abort_flag) {
        // drain: every slot whose copy was issued must land before the CTA exits
        volatile int never = 0;
        for (int i = (issued > C::STAGES ? issued - C::STAGES : 0); i < issued; ++i)
          mbar_wait_bounded(&full[i % C::STAGES], (uint32_t)(i / C::STAGES) & 1u, &never, 200000000ull);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3(BM, BN);
      int i = 0;
      for (; i < nkb; ++i) {
        const int s = i % C::STAGES;
        const uint32_t ph = (uint32_t)(i / C::STAGES) & 1u;
        if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t wbase = smem_u32(smem + s * C::STAGE_BYTES);
        const uint64_t dw = umma_desc_sw128(wbase);
        const uint64_t da = umma_desc_sw128(wbase + W_TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < BK / UMMA_K; ++kk) {
          // +32 bytes per K step inside the swizzle atom = +2 in the encoded address
          umma_f8f6f4(tmem, dw + 2 * kk, da + 2 * kk, idesc, (i | kk) != 0);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(accum);  // fires once every MMA issued above has completed
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    const int n = n0 + row;
    const bool ok = mbar_wait_bounded(accum, 0, abort_flag);
    tc_fence_after();
    pdl_launch();
    if (!ok) *abort_flag = 1;
    const bool live = ok && !*abort_flag;
    const float sw = args.w_per_col ? (n < args.N ? args.w_scale[n] : 0.f) : args.w_scale[0];
    const float sa0 = args.a_scale[0];
    const uint32_t lane_base = tmem + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      float v[16];
      tmem_ld16(lane_base + (uint32_t)c, v);  // warp-collective: every lane executes it
      if (args.epilogue == FFB_EPI_SWIGLU) {
        // Rows 64..127 hold the up projections of gate rows 0..63 of this tile.  Both named
        // barriers run unconditionally so the 128 epilogue threads always meet them.
        if (live && row >= 64) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c + j;
            const float sa = args.a_per_row ? (m < args.M ? args.a_scale[m] : 0.f) : sa0;
            xchg[(row - 64) * 16 + j] = round_bf(v[j] * sa * sw);
          }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(EPI_THREADS) : "memory");
        if (live && row < 64) {
          const int ch = ft * 64 + row;
          const int ldo = args.N / 2;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + c + j;
            if (m < args.M) {
              const float sa = args.a_per_row ? args.a_scale[m] : sa0;
              const float g = round_bf(v[j] * sa * sw);
              const float u = xchg[row * 16 + j];
              const float act = round_bf(__fdiv_rn(g, 1.f + expf(-g)));
              args.out[(size_t)m * ldo + ch] = f2bf(act * u);
            }
          }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(EPI_THREADS) : "memory");
      } else if (!live) {
        continue;
      } else if (args.epilogue == FFB_EPI_F32_PARTIAL) {
        float* dst = args.ws + (size_t)ks * args.M * args.N;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + c + j;
          if (m < args.M && n < args.N) {
            const float sa = args.a_per_row ? args.a_scale[m] : sa0;
            dst[(size_t)m * args.N + n] = v[j] * sa * sw;
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + c + j;
          if (m < args.M && n < args.N) {
            const float sa = args.a_per_row ? args.a_scale[m] : sa0;
            args.out[(size_t)m * args.N + n] = f2bf(v[j] * sa * sw);
          }
        }
      }
    }
  }

  if (warp == 1 && lane == 0 && *abort_flag) {
    // MMAs already issued must finish before their TMEM is released
    volatile int never = 0;
    mbar_wait_bounded(accum, 0, &never, 200000000ull);
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

template <int BN>
int launch_bn(const CUtensorMap& tw, const uint8_t* a8, const GemmArgs& ga, cudaStream_t stream) {
  using C = Cfg<BN>;
  CUtensorMap ta;
  int rc = ffb::make_tmap_2d(&ta, a8, (uint64_t)ga.M, (uint64_t)ga.K, (uint64_t)ga.K, BN, BK, 1);
  if (rc) return rc;
  static bool attr_set = false;  // per process; the attribute is per function
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(fp8_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_fp8_gemm: smem attribute: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  GemmArgs a = ga;
  const int grid = (ga.N / BM) * ga.splits * ga.n_ttiles;
  cudaError_t e = ffb::launch(fp8_gemm_kernel<BN>, dim3(grid), dim3(192), C::SMEM, stream, tw, ta, a);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_fp8_gemm: launch: %s", cudaGetErrorString(e));
  return FFB_OK;
}

}  // namespace

namespace ffb {
// Token tile chosen when the caller passes 0: the fewest tiles of <= 256 tokens, each a
// multiple of 16 (32 above 16) so that one tcgen05.mma covers it.
int pick_token_tile(int M) {
  if (M <= 16) return 16;
  const int nt = (M + 255) / 256;
  int bn = (M + nt - 1) / nt;
  bn = (bn + 31) / 32 * 32;
  return bn > 256 ? 256 : bn;
}
}  // namespace ffb

extern "C" int ffb_fp8_gemm(const uint8_t* a8, const float* a_scale, int a_per_row, const uint8_t* w8,
                            const float* w_scale, int w_per_col, int epilogue, uint16_t* out, float* ws, int splits,
                            int token_tile, int M, int N, int K, void* stream) {
  FFB_REQUIRE(a8 && w8 && a_scale && w_scale, "ffb_fp8_gemm: NULL operand");
  FFB_REQUIRE(M > 0 && N > 0 && K > 0, "ffb_fp8_gemm: bad shape M=%d N=%d K=%d", M, N, K);
  FFB_REQUIRE(N % BM == 0, "ffb_fp8_gemm: N=%d must be a multiple of 128", N);
  FFB_REQUIRE(K % 16 == 0, "ffb_fp8_gemm: K=%d must be a multiple of 16", K);
  FFB_REQUIRE(ffb::aligned(a8, 16) && ffb::aligned(w8, 16), "ffb_fp8_gemm: operands must be 16-byte aligned");
  FFB_REQUIRE(epilogue == FFB_EPI_BF16 || epilogue == FFB_EPI_F32_PARTIAL || epilogue == FFB_EPI_SWIGLU,
              "ffb_fp8_gemm: unknown epilogue %d", epilogue);
  const int nkb = (K + BK - 1) / BK;
  if (epilogue == FFB_EPI_F32_PARTIAL) {
    FFB_REQUIRE(ws != nullptr, "ffb_fp8_gemm: F32_PARTIAL needs ws");
    FFB_REQUIRE(splits >= 1 && splits <= nkb, "ffb_fp8_gemm: splits=%d outside [1, %d]", splits, nkb);
  } else {
    FFB_REQUIRE(out != nullptr, "ffb_fp8_gemm: out is NULL");
    FFB_REQUIRE(splits == 1, "ffb_fp8_gemm: splits must be 1 unless the epilogue is F32_PARTIAL");
  }
  int bn = token_tile > 0 ? token_tile : ffb::pick_token_tile(M);
  GemmArgs ga;
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
  ga.n_ttiles = (M + bn - 1) / bn;
  CUtensorMap tw;
  int rc = ffb::make_tmap_2d(&tw, w8, (uint64_t)N, (uint64_t)K, (uint64_t)K, BM, BK, 1);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (bn) {
    case 16: return launch_bn<16>(tw, a8, ga, s);
    case 32: return launch_bn<32>(tw, a8, ga, s);
    case 64: return launch_bn<64>(tw, a8, ga, s);
    case 96: return launch_bn<96>(tw, a8, ga, s);
    case 128: return launch_bn<128>(tw, a8, ga, s);
    case 160: return launch_bn<160>(tw, a8, ga, s);
    case 192: return launch_bn<192>(tw, a8, ga, s);
    case 224: return launch_bn<224>(tw, a8, ga, s);
    case 256: return launch_bn<256>(tw, a8, ga, s);
    default: return ffb::fail(FFB_EUNSUPPORTED, "ffb_fp8_gemm: token tile %d not built (16,32,64..256 step 32)", bn);
  }
}
