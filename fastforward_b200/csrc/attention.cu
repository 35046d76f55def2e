// Causal GQA attention for head_dim 128: the pick-row tail (selected query rows) and
// prefill with unaligned outputs here; the full causal prefill goes to the tcgen05 kernel
// of attention_tc.cu.
//
// Semantics of the reference kernel (_legacy/limit_kernels.py:8-33): scores in fp32,
// scaled by 1/sqrt(128); online softmax over key blocks (running max, rescaled
// accumulator); the probabilities are cast to bf16 before the P.V product; output
// bf16(acc / den).  Keys n > position are masked (position = query index, or the
// explicit `positions` of the tail's selected rows).
//
// Tiling: one CTA = one query head x 64 query rows (4 warps x 16 rows); key/value blocks
// of 64 rows double-buffered in shared memory through cp.async (XOR-swizzled 16-byte
// chunks so the ldmatrix reads are conflict-free); S = Q.K^T and O += P.V on the
// bf16 mma.sync tensor-core path with fp32 accumulation; P stays in registers.
#include "common.cuh"
#include "pdl.cuh"

namespace {

constexpr int D = 128;
constexpr int BMQ = 64;
constexpr int BNK = 64;
constexpr int TILE_BYTES = 64 * D * 2;  // 16 KB
constexpr int SMEM = TILE_BYTES * 5;    // Q + 2 x (K, V)

__device__ __forceinline__ uint32_t swz(int row, int chunk) {  // byte offset inside a [64 x 128] bf16 tile
  return (uint32_t)(row * 256 + ((chunk ^ (row & 7)) << 4));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  return (uint32_t)f2bf(lo) | ((uint32_t)f2bf(hi) << 16);
}

// Loads rows [r0, r0+64) of a [rows x 128] bf16 matrix into a swizzled tile; rows >= nrows are zero.
__device__ __forceinline__ void load_tile(uint32_t tile, const uint16_t* src, int r0, int nrows) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int idx = threadIdx.x + i * 128;  // 1024 chunks of 16 bytes
    const int r = idx >> 4, c = idx & 15;
    const int gr = r0 + r;
    const bool ok = gr < nrows;
    cp_async16(tile + swz(r, c), src + (size_t)(ok ? gr : 0) * D + c * 8, ok);
  }
}

struct AttnArgs {
  const uint16_t* q;
  const uint16_t* k;
  const uint16_t* v;
  const int64_t* positions;
  const int* key_lo;  // per query row: its lowest visible key, or NULL = 0
  int q_gather;
  uint16_t* out;
  int S, T, HQ, HK;
  float scale_log2;  // scale * log2(e)
};

__global__ void __launch_bounds__(128) attention_kernel(const AttnArgs p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sbase = smem_u32(smem);
  const uint32_t sQ = sbase, sK0 = sbase + TILE_BYTES, sV0 = sbase + 2 * TILE_BYTES;
  const uint32_t sK1 = sbase + 3 * TILE_BYTES, sV1 = sbase + 4 * TILE_BYTES;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int h = blockIdx.y, kvh = h / (p.HQ / p.HK);
  const int q0 = blockIdx.x * BMQ;

  pdl_wait();

  pdl_launch();
  // positions of this thread's two rows and the key range the block needs
  const int ra = q0 + warp * 16 + g, rb = ra + 8;
  auto pos_of = [&](int r) -> int {
    if (r >= p.S) return -1;
    return p.positions ? (int)p.positions[r] : r;
  };
  const int pa = pos_of(ra), pb = pos_of(rb);
  const int loa = p.key_lo && ra < p.S ? p.key_lo[ra] : 0, lob = p.key_lo && rb < p.S ? p.key_lo[rb] : 0;
  // first key block: the lowest key any row of the block can see
  int kstart = 0;
  if (p.key_lo) {
    int mn = 1 << 30;
    for (int r = q0 + threadIdx.x; r < min(q0 + BMQ, p.S); r += 128) mn = min(mn, p.key_lo[r]);
    __shared__ int red_lo[4];
    mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, 16));
    mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, 8));
    mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, 4));
    mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, 2));
    mn = min(mn, __shfl_xor_sync(0xffffffffu, mn, 1));
    if (lane == 0) red_lo[warp] = mn;
    __syncthreads();
    kstart = max(0, min(min(red_lo[0], red_lo[1]), min(red_lo[2], red_lo[3])));
  }
  int kend;
  if (p.positions) {
    int mx = -1;
    for (int r = q0 + threadIdx.x; r < min(q0 + BMQ, p.S); r += 128) mx = max(mx, (int)p.positions[r]);
    __shared__ int red[4];
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    kend = min(p.T, max(max(red[0], red[1]), max(red[2], red[3])) + 1);
  } else {
    kend = min(p.T, min(q0 + BMQ, p.S));
  }
  const int blk0 = min(kstart / BNK, (kend + BNK - 1) / BNK);
  const int nblk = (kend + BNK - 1) / BNK - blk0;  // key blocks visited, from key blk0 * BNK

  const uint16_t* kh = p.k + (size_t)kvh * p.T * D;
  const uint16_t* vh = p.v + (size_t)kvh * p.T * D;
  if (p.q_gather) {
    // query row s is row positions[s] of the full [HQ, T, 128] projection
    const uint16_t* qh = p.q + (size_t)h * p.T * D;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int idx = threadIdx.x + i * 128;
      const int r = idx >> 4, c = idx & 15;
      const int gr = q0 + r;
      const bool ok = gr < p.S;
      int src_row = ok ? (int)p.positions[gr] : 0;
      if (src_row < 0 || src_row >= p.T) src_row = 0;  // keeps the read in bounds for a bad index
      cp_async16(sQ + swz(r, c), qh + (size_t)src_row * D + c * 8, ok);
    }
  } else {
    load_tile(sQ, p.q + (size_t)h * p.S * D, q0, p.S);
  }
  if (nblk > 0) {
    load_tile(sK0, kh, blk0 * BNK, p.T);
    load_tile(sV0, vh, blk0 * BNK, p.T);
  }
  cp_commit();

  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float ma = -INFINITY, mb = -INFINITY, la = 0.f, lb = 0.f;
  uint32_t qf[8][4];

  for (int blk = 0; blk < nblk; ++blk) {
    const uint32_t sK = (blk & 1) ? sK1 : sK0, sV = (blk & 1) ? sV1 : sV0;
    if (blk + 1 < nblk) {
      load_tile((blk & 1) ? sK0 : sK1, kh, (blk0 + blk + 1) * BNK, p.T);
      load_tile((blk & 1) ? sV0 : sV1, vh, (blk0 + blk + 1) * BNK, p.T);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (blk == 0) {
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int r = warp * 16 + (lane & 15), c = kk * 2 + (lane >> 4);
        ldsm_x4(sQ + swz(r, c), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    // S = Q K^T : 16 rows x 64 keys per warp
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {  // pairs of 8-key tiles
        const int key = jp * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = kk * 2 + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(sK + swz(key, c), b0, b1, b2, b3);
        mma_bf16(s[2 * jp], qf[kk], b0, b1);
        mma_bf16(s[2 * jp + 1], qf[kk], b2, b3);
      }
    }
    // mask + online softmax (base-2 exponent of score * scale * log2 e)
    float bmax_a = -INFINITY, bmax_b = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int key = (blk0 + blk) * BNK + j * 8 + 2 * t4 + e;
        float va = s[j][e] * p.scale_log2, vb = s[j][2 + e] * p.scale_log2;
        if (key > pa || key >= p.T || key < loa) va = -INFINITY;
        if (key > pb || key >= p.T || key < lob) vb = -INFINITY;
        s[j][e] = va;
        s[j][2 + e] = vb;
        bmax_a = fmaxf(bmax_a, va);
        bmax_b = fmaxf(bmax_b, vb);
      }
    }
    bmax_a = fmaxf(bmax_a, __shfl_xor_sync(0xffffffffu, bmax_a, 1));
    bmax_a = fmaxf(bmax_a, __shfl_xor_sync(0xffffffffu, bmax_a, 2));
    bmax_b = fmaxf(bmax_b, __shfl_xor_sync(0xffffffffu, bmax_b, 1));
    bmax_b = fmaxf(bmax_b, __shfl_xor_sync(0xffffffffu, bmax_b, 2));
    const float na = fmaxf(ma, bmax_a), nb = fmaxf(mb, bmax_b);
    const float base_a = na == -INFINITY ? 0.f : na, base_b = nb == -INFINITY ? 0.f : nb;
    const float alpha_a = exp2f(ma - base_a), alpha_b = exp2f(mb - base_b);
    ma = na;
    mb = nb;
    la *= alpha_a;
    lb *= alpha_b;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      o[i][0] *= alpha_a;
      o[i][1] *= alpha_a;
      o[i][2] *= alpha_b;
      o[i][3] *= alpha_b;
    }
    uint32_t pf[4][4];  // P as A fragments for the 4 key steps of 16
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = exp2f(s[j][0] - base_a), p1 = exp2f(s[j][1] - base_a);
      const float p2 = exp2f(s[j][2] - base_b), p3 = exp2f(s[j][3] - base_b);
      la += p0 + p1;
      lb += p2 + p3;
      pf[j >> 1][(j & 1) * 2 + 0] = pack_bf2(p0, p1);
      pf[j >> 1][(j & 1) * 2 + 1] = pack_bf2(p2, p3);
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t a[4] = {pf[kk][0], pf[kk][1], pf[kk][2], pf[kk][3]};
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {  // pairs of 8-wide d tiles
        const int key = kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = dp * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sV + swz(key, c), b0, b1, b2, b3);
        mma_bf16(o[2 * dp], a, b0, b1);
        mma_bf16(o[2 * dp + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_wait<0>();
  
  la += __shfl_xor_sync(0xffffffffu, la, 1);
  la += __shfl_xor_sync(0xffffffffu, la, 2);
  lb += __shfl_xor_sync(0xffffffffu, lb, 1);
  lb += __shfl_xor_sync(0xffffffffu, lb, 2);
  const int ld = p.HQ * D;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int d = i * 8 + 2 * t4;
    if (ra < p.S) {
      const float inv = 1.f / la;
      *reinterpret_cast<uint32_t*>(p.out + (size_t)ra * ld + h * D + d) = pack_bf2(o[i][0] * inv, o[i][1] * inv);
    }
    if (rb < p.S) {
      const float inv = 1.f / lb;
      *reinterpret_cast<uint32_t*>(p.out + (size_t)rb * ld + h * D + d) = pack_bf2(o[i][2] * inv, o[i][3] * inv);
    }
  }
}

}  // namespace

int ffb_attention_tc(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int* key_lo, void* out, int T,
                     int HQ, int HK, float scale, float out_inv, cudaStream_t stream);

extern "C" int ffb_attention_segmented(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                       const int64_t* positions, int q_gather, const int* key_lo, uint16_t* out, int S,
                                       int T, int HQ, int HK, float scale, void* stream) {
  FFB_REQUIRE(q && k && v && out, "ffb_attention: NULL pointer");
  FFB_REQUIRE(S > 0 && T > 0 && HQ > 0 && HK > 0 && HQ % HK == 0, "ffb_attention: bad shape S=%d T=%d HQ=%d HK=%d", S,
              T, HQ, HK);
  FFB_REQUIRE(positions || S <= T, "ffb_attention: causal prefill needs S <= T");
  FFB_REQUIRE(!q_gather || positions, "ffb_attention: q_gather needs positions");
  FFB_REQUIRE(ffb::aligned(q, 16) && ffb::aligned(k, 16) && ffb::aligned(v, 16) && ffb::aligned(out, 4),
              "ffb_attention: alignment");
  FFB_REQUIRE(!key_lo || ffb::aligned(key_lo, 4), "ffb_attention: key_lo alignment");
  if (!positions && S == T && ffb::aligned(out, 16))  // causal prefill: the tcgen05 kernel
    return ffb_attention_tc(q, k, v, key_lo, out, T, HQ, HK, scale, 0.f, (cudaStream_t)stream);
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
    if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_attention: %s", cudaGetErrorString(e));
    attr = true;
  }
  AttnArgs a = {q, k, v, positions, key_lo, q_gather, out, S, T, HQ, HK, scale * 1.4426950408889634f};
  cudaError_t e = ffb::launch(attention_kernel, dim3((S + BMQ - 1) / BMQ, HQ), dim3(128), SMEM,
                              (cudaStream_t)stream, a);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_attention: %s", cudaGetErrorString(e));
  return FFB_OK;
}

extern "C" int ffb_attention_fp8(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int* key_lo,
                                 float out_inv, uint8_t* out8, int T, int HQ, int HK, float scale, void* stream) {
  FFB_REQUIRE(q && k && v && out8, "ffb_attention_fp8: NULL pointer");
  FFB_REQUIRE(T > 0 && HQ > 0 && HK > 0 && HQ % HK == 0, "ffb_attention_fp8: bad shape T=%d HQ=%d HK=%d", T, HQ, HK);
  FFB_REQUIRE(out_inv > 0.f, "ffb_attention_fp8: out_inv must be positive");
  FFB_REQUIRE(ffb::aligned(q, 16) && ffb::aligned(k, 16) && ffb::aligned(v, 16) && ffb::aligned(out8, 16),
              "ffb_attention_fp8: alignment");
  FFB_REQUIRE(!key_lo || ffb::aligned(key_lo, 4), "ffb_attention_fp8: key_lo alignment");
  return ffb_attention_tc(q, k, v, key_lo, out8, T, HQ, HK, scale, out_inv, (cudaStream_t)stream);
}

extern "C" int ffb_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int64_t* positions,
                             int q_gather, uint16_t* out, int S, int T, int HQ, int HK, float scale, void* stream) {
  return ffb_attention_segmented(q, k, v, positions, q_gather, nullptr, out, S, T, HQ, HK, scale, stream);
}
