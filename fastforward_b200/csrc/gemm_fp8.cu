// FP8 e4m3 W8A8 linear on the sm_100a tensor cores (tcgen05, kind::f8f6f4).
//
// Replaces the reference's quantiser + torch._scaled_mm pair
// (_family/depth_fp8.py:22-26, _legacy/fp8_private.py:29-38).
//
// Orientation ("swap AB"): the weight tile is the 128-row UMMA A operand and the tokens
// are the UMMA N dimension, so a tile is 128 output features x BN tokens; for a prefill
// of T <= 256 tokens every weight byte streams from HBM once.  D[feature, token]
// accumulates in tensor memory (fp32).
//
// Persistent kernel, one CTA per SM, tiles assigned round-robin.  Roles (320 threads):
//   warp 0      TMA producer: weight tile + token tile per 128-byte K block into a ring
//               of STAGES shared-memory slots (full[s] / empty[s] mbarriers);
//   warp 1      TMEM allocator + single-thread MMA issuer; two accumulator buffers in
//               TMEM so the MMAs of tile i+1 overlap the epilogue of tile i
//               (tmem_full[b] / tmem_empty[b]);
//   warps 2..9  epilogue: per 32-token chunk, the 8 warps load the fp32 accumulators
//               (warp w reads TMEM lanes 32*(w%4).. and columns 16*((w-2)/4)..), apply
//               the per-token and per-feature scales, stage the chunk transposed in shared
//               memory, then write it token-major with 16-byte stores (bf16 / fp32 split-K
//               partial / fused SwiGLU).
// Every wait is bounded (mbar_wait_bounded); a timeout sets the CTA abort flag and the
// device error word; all roles then unwind, in-flight copies and MMAs drain, TMEM is
// released.  The epilogue's named barriers are reached by all 256 epilogue threads on
// every path (one elected thread waits on the accumulator barrier and broadcasts).
#include "common.cuh"
#include "pdl.cuh"

namespace {

constexpr int BM = 128;      // features per tile (UMMA M)
constexpr int BK = 128;      // K bytes per stage (one 128-byte swizzle atom row)
constexpr int UMMA_K = 32;   // K per tcgen05.mma for 8-bit operands
constexpr int W_TILE_BYTES = BM * BK;
constexpr int EPI_WARPS = 8;
constexpr int EPI_THREADS = EPI_WARPS * 32;
constexpr int THREADS = 64 + EPI_THREADS;
constexpr int CHUNK = 32;                 // tokens per epilogue chunk
constexpr int STG_STRIDE = BM + 4;        // fp32 words per staged token row (padding vs bank conflicts)
constexpr int STG_BYTES = CHUNK * STG_STRIDE * 4;
constexpr int SMEM_LIMIT = 232448;

__host__ __device__ constexpr int tmem_cols_for(int bn) {
  return bn <= 32 ? 32 : bn <= 64 ? 64 : bn <= 128 ? 128 : 256;
}
template <int BN>
struct Cfg {
  static constexpr int A_TILE_BYTES = BN * BK;
  static constexpr int STAGE_BYTES = W_TILE_BYTES + A_TILE_BYTES;
  static constexpr int FIXED = 2 * STG_BYTES + 512 + 1024;  // staging, barriers, alignment slack
  static constexpr int FIT = (SMEM_LIMIT - FIXED) / STAGE_BYTES;
  static constexpr int STAGES = FIT > 8 ? 8 : FIT;
  static constexpr int SMEM = STAGES * STAGE_BYTES + FIXED;
  static constexpr int ACC_COLS = tmem_cols_for(BN);  // one accumulator buffer
  static constexpr int TMEM_COLS = 2 * ACC_COLS;
  static_assert(STAGES >= 2, "shared memory too small for two stages");
};

struct GemmArgs {
  const float* a_scale;
  const float* w_scale;
  uint16_t* out;
  float* ws;
  int a_per_row, w_per_col, epilogue;
  int M, N, K, n_ttiles, splits, n_tiles;
};

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(EPI_THREADS) : "memory"); }

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
    fp8_gemm_kernel(const __grid_constant__ CUtensorMap tmap_w, const __grid_constant__ CUtensorMap tmap_a,
                    const GemmArgs args) {
  using C = Cfg<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* stg = reinterpret_cast<float*>(smem + C::STAGES * C::STAGE_BYTES);  // 2 staging buffers
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES + 2 * STG_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* tfull = empty + C::STAGES;  // [2]
  uint64_t* tempty = tfull + 2;         // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* epi_ok = abort_flag + 1;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nkb_total = (args.K + BK - 1) / BK;

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
    *epi_ok = 1;
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

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first(), pol_a = policy_evict_last();
      // The weights do not depend on the previous kernel: the weight tiles of the first
      // ring pass are requested before the programmatic-launch wait, so their HBM latency
      // overlaps the tail of the kernel that produces this GEMM's activations.
      int pre = 0;
      {
        const int t = blockIdx.x;
        if (t < args.n_tiles) {
          const int rest = t / args.n_ttiles;
          const int ks = rest % args.splits, ft = rest / args.splits;
          const int kb0 = (int)((long long)ks * nkb_total / args.splits);
          const int kb1 = (int)((long long)(ks + 1) * nkb_total / args.splits);
          pre = kb1 - kb0 < C::STAGES ? kb1 - kb0 : C::STAGES;
          for (int i = 0; i < pre; ++i) {
            mbar_arrive_expect_tx(&full[i], C::STAGE_BYTES);
            tma_load_2d(smem + i * C::STAGE_BYTES, &tmap_w, &full[i], (kb0 + i) * BK, ft * BM, pol_w);
          }
        }
      }
      pdl_wait();
      int it = 0;
      for (int t = blockIdx.x; t < args.n_tiles && !*abort_flag; t += gridDim.x) {
        const int tt = t % args.n_ttiles, rest = t / args.n_ttiles;
        const int ks = rest % args.splits, ft = rest / args.splits;
        const int kb0 = (int)((long long)ks * nkb_total / args.splits);
        const int kb1 = (int)((long long)(ks + 1) * nkb_total / args.splits);
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
          uint8_t* st = smem + s * C::STAGE_BYTES;
          if (it < pre) {  // weight half already in flight; add the activation half
            tma_load_2d(st + W_TILE_BYTES, &tmap_a, &full[s], kb * BK, tt * BN, pol_a);
            continue;
          }
          if (!mbar_wait_bounded(&empty[s], ph ^ 1u, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
          tma_load_2d(st, &tmap_w, &full[s], kb * BK, ft * BM, pol_w);
          tma_load_2d(st + W_TILE_BYTES, &tmap_a, &full[s], kb * BK, tt * BN, pol_a);
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
    pdl_wait();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_e4m3(BM, BN);
      int it = 0, lt = 0;
      for (int t = blockIdx.x; t < args.n_tiles && !*abort_flag; t += gridDim.x, ++lt) {
        const int rest = t / args.n_ttiles;
        const int ks = rest % args.splits;
        const int kb0 = (int)((long long)ks * nkb_total / args.splits);
        const int kb1 = (int)((long long)(ks + 1) * nkb_total / args.splits);
        const int buf = lt & 1;
        const uint32_t use = (uint32_t)(lt >> 1);
        if (!mbar_wait_bounded(&tempty[buf], (use & 1u) ^ 1u, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * C::ACC_COLS);
        bool ok = true;
        for (int kb = kb0; kb < kb1; ++kb, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (uint32_t)(it / C::STAGES) & 1u;
          if (!mbar_wait_bounded(&full[s], ph, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t wbase = smem_u32(smem + s * C::STAGE_BYTES);
          const uint64_t dw = umma_desc_sw128(wbase);
          const uint64_t da = umma_desc_sw128(wbase + W_TILE_BYTES);
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk)  // +32 bytes per K step = +2 encoded
            umma_f8f6f4(acc, dw + 2 * kk, da + 2 * kk, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
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
    const int ew = warp - 2;            // 0..7
    const int q = warp & 3;             // TMEM lane quarter this warp may access
    const int hlf = ew >> 2;            // which 16 columns of a 32-token chunk
    const int etid = tid - 64;          // 0..255
    const int feat = q * 32 + lane;     // feature row this thread loads
    int lt = 0;
    for (int t = blockIdx.x; t < args.n_tiles; t += gridDim.x, ++lt) {
      const int tt = t % args.n_ttiles, rest = t / args.n_ttiles;
      const int ks = rest % args.splits, ft = rest / args.splits;
      const int n0 = ft * BM, m0 = tt * BN;
      const int buf = lt & 1;
      const uint32_t use = (uint32_t)(lt >> 1);
      if (etid == 0) *epi_ok = mbar_wait_bounded(&tfull[buf], use & 1u, abort_flag) && !*abort_flag;
      epi_bar();
      if (!*epi_ok) break;  // uniform: every epilogue thread reads the same flag after the barrier
      tc_fence_after();
      const int n = n0 + feat;
      const float sw = args.w_per_col ? args.w_scale[n] : args.w_scale[0];
      const float sa0 = args.a_scale[0];
      const uint32_t acc = tmem + (uint32_t)(buf * C::ACC_COLS) + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = 0, ci = 0; c < BN; c += CHUNK, ++ci) {
        float* sb = stg + (ci & 1) * (CHUNK * STG_STRIDE);
        const int col = c + hlf * 16;
        if (col < BN) {  // warp-uniform
          float v[16];
          tmem_ld16(acc + (uint32_t)col, v);
          const bool swiglu = args.epilogue == FFB_EPI_SWIGLU;
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = m0 + col + j;
            const float sa = args.a_per_row ? (m < args.M ? args.a_scale[m] : 0.f) : sa0;
            float y = v[j] * sa * sw;
            if (swiglu) y = round_bf(y);  // the linear's bf16 output feeds the activation
            sb[(hlf * 16 + j) * STG_STRIDE + feat] = y;
          }
        }
        epi_bar();
        // token-major output of the staged [32 tokens x 128 features] chunk
        const int tok = etid & 31, grp = etid >> 5;  // warp grp handles one feature group
        const int m = m0 + c + tok;
        if (c + tok < BN && m < args.M) {
          const float* row = sb + tok * STG_STRIDE;
          if (args.epilogue == FFB_EPI_SWIGLU) {
            // tile rows 0..63 are gate channels ft*64 + r, rows 64..127 the matching up rows
            float g[8], u[8];
            *reinterpret_cast<float4*>(g) = *reinterpret_cast<const float4*>(row + grp * 8);
            *reinterpret_cast<float4*>(g + 4) = *reinterpret_cast<const float4*>(row + grp * 8 + 4);
            *reinterpret_cast<float4*>(u) = *reinterpret_cast<const float4*>(row + 64 + grp * 8);
            *reinterpret_cast<float4*>(u + 4) = *reinterpret_cast<const float4*>(row + 64 + grp * 8 + 4);
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              const float a0 = round_bf(__fdiv_rn(g[e], 1.f + expf(-g[e])));
              const float a1 = round_bf(__fdiv_rn(g[e + 1], 1.f + expf(-g[e + 1])));
              o[e / 2] = (uint32_t)f2bf(a0 * u[e]) | ((uint32_t)f2bf(a1 * u[e + 1]) << 16);
            }
            uint16_t* dst = args.out + (size_t)m * (args.N / 2) + ft * 64 + grp * 8;
            *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
          } else if (args.epilogue == FFB_EPI_F32_PARTIAL) {
            float* dst = args.ws + ((size_t)ks * args.M + m) * args.N + n0 + grp * 16;
#pragma unroll
            for (int e = 0; e < 16; e += 4)
              *reinterpret_cast<float4*>(dst + e) = *reinterpret_cast<const float4*>(row + grp * 16 + e);
          } else {
            float f[16];
#pragma unroll
            for (int e = 0; e < 16; e += 4)
              *reinterpret_cast<float4*>(f + e) = *reinterpret_cast<const float4*>(row + grp * 16 + e);
            uint32_t o[8];
#pragma unroll
            for (int e = 0; e < 16; e += 2) o[e / 2] = (uint32_t)f2bf(f[e]) | ((uint32_t)f2bf(f[e + 1]) << 16);
            uint16_t* dst = args.out + (size_t)m * args.N + n0 + grp * 16;
            *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
            *reinterpret_cast<uint4*>(dst + 8) = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
      }
      // this warp's TMEM reads of the buffer are complete (tcgen05.ld waited): release it
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
    }
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
int launch_bn(const CUtensorMap& tw, const uint8_t* a8, const GemmArgs& ga, int max_ctas, cudaStream_t stream) {
  using C = Cfg<BN>;
  CUtensorMap ta;
  int rc = ffb::make_tmap_2d(&ta, a8, (uint64_t)ga.M, (uint64_t)ga.K, (uint64_t)ga.K, BN, BK, 1);
  if (rc) return rc;
  static bool attr_set = false;  // the attribute is per function (one device per process here)
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(fp8_gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
    if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_fp8_gemm: smem attribute: %s", cudaGetErrorString(e));
    attr_set = true;
  }
  int grid = ga.n_tiles < num_sms() ? ga.n_tiles : num_sms();
  if (max_ctas > 0 && grid > max_ctas) grid = max_ctas;
  cudaError_t e = ffb::launch(fp8_gemm_kernel<BN>, dim3(grid), dim3(THREADS), C::SMEM, stream, tw, ta, ga);
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
    FFB_REQUIRE(ws != nullptr && ffb::aligned(ws, 16), "ffb_fp8_gemm: F32_PARTIAL needs a 16-byte aligned ws");
    FFB_REQUIRE(splits >= 1 && splits <= nkb, "ffb_fp8_gemm: splits=%d outside [1, %d]", splits, nkb);
  } else {
    FFB_REQUIRE(out != nullptr && ffb::aligned(out, 16), "ffb_fp8_gemm: out must be non-NULL, 16-byte aligned");
    FFB_REQUIRE(splits == 1, "ffb_fp8_gemm: splits must be 1 unless the epilogue is F32_PARTIAL");
  }
  const int bn = token_tile > 0 ? token_tile : ffb::pick_token_tile(M);
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
  ga.n_tiles = (N / BM) * splits * ga.n_ttiles;
  CUtensorMap tw;
  int rc = ffb::make_tmap_2d(&tw, w8, (uint64_t)N, (uint64_t)K, (uint64_t)K, BM, BK, 1);
  if (rc) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (bn) {
    case 16: return launch_bn<16>(tw, a8, ga, 0, s);
    case 32: return launch_bn<32>(tw, a8, ga, 0, s);
    case 64: return launch_bn<64>(tw, a8, ga, 0, s);
    case 96: return launch_bn<96>(tw, a8, ga, 0, s);
    case 128: return launch_bn<128>(tw, a8, ga, 0, s);
    case 160: return launch_bn<160>(tw, a8, ga, 0, s);
    case 192: return launch_bn<192>(tw, a8, ga, 0, s);
    case 224: return launch_bn<224>(tw, a8, ga, 0, s);
    case 256: return launch_bn<256>(tw, a8, ga, 0, s);
    default: return ffb::fail(FFB_EUNSUPPORTED, "ffb_fp8_gemm: token tile %d not built (16,32,64..256 step 32)", bn);
  }
}
