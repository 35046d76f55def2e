// Causal GQA prefill attention (head_dim 128) on the sm_100a tensor cores: TMA-fed
// tcgen05 MMAs with the score and output tiles in tensor memory.
//
// Semantics of the reference kernel (_legacy/limit_kernels.py:8-33, BLOCK_N = 64): scores
// in fp32 scaled by 1/sqrt(128); online softmax over 64-key blocks (running max m,
// denominator l = l * alpha + sum(p), accumulator acc = acc * alpha + P.V with
// alpha = exp(m_old - m_new)); P cast to bf16 before its product with V; output
// bf16(acc / l).  Keys past the query's position (and past T) are masked.  The reference
// leaves the exponential (tl.exp) and the reduction orders to its compiler; this kernel
// fixes every one of them so that its output is a function of its inputs alone, restated
// operation for operation by the oracle (oracle/attn.c):
//   x = fp32(s * scale * log2 e); m_new = max(m, block max); base = m_new;
//   alpha = exp2_poly(m - base), p = exp2_poly(x - base) (this file's polynomial
//   exponential, on the FMA pipe); each of a row's four parts keeps its denominator share
//   l = fma(l, alpha, psum) with psum its 16 keys summed pairwise in key order;
//   o = fma(o, alpha, O_j); l = ((l0 + l1) + l2) + l3; the final quotient is correctly
//   rounded before the bf16 cast.
//
// One CTA = 128 query rows of one head (the M of the MMA); 576 threads:
//   warp 0     TMA producer: the Q tile once ([128 x 128] as two 64-column swizzled
//              halves), K and V blocks of 64 keys into a ring of KV_STAGES slots;
//   warp 1     TMEM allocator + single-thread MMA issuer:
//                S_j = Q . K_j^T  (M 128, N 64, 8 x K16, both operands K-major) -> TMEM;
//                O_j = P_j . V_j  (M 128, N 128, 4 x K16; V read MN-major straight from
//                                  its row-major [key][d] tile) -> TMEM;
//   warps 2..17 softmax, four threads per query row (TMEM lane quarter = warp % 4; the four
//              warps of a quarter are its parts 0..3): part p reads keys [16p, 16p + 16) of
//              the block's 64 scores, the four exchange their row maxima through shared
//              memory, each writes its 16 bf16 P values into the swizzled [128 x 64] P tile,
//              keeps its own part of the denominator (same alpha) and folds output
//              columns [32p, 32p + 32) of the previous block's O into fp32 registers
//              (o = o * alpha + O, one block late).  At the end the rows' quotients are
//              staged in shared memory (the P tiles, by then free) and leave by TMA store.
// S, P and O are double-buffered: the MMA warp issues S_{j+2} as soon as the softmax has
// read S_j and P_j . V_j as soon as P_j is written, so the tensor core works on the next
// blocks while the softmax runs.  Barriers: q_full, kv_full/kv_empty[stage],
// s_full/s_free[2], p_full[2], o_full[2].  Every wait is bounded; a timeout sets the
// abort flag and the device error word, and TMEM is released.
#include "common.cuh"
#include "pdl.cuh"

#include <string.h>

namespace {

constexpr int D = 128;
constexpr int BM = 128;             // query rows per CTA (UMMA M)
constexpr int BN = 64;              // keys per block (the reference's BLOCK_N)
constexpr int KV_STAGES = 3;
constexpr int Q_HALF = BM * 128;    // one 64-column half of the Q tile: 16 KB
constexpr int KV_HALF = BN * 128;   // one 64-column half of a K or V block: 8 KB
constexpr int STAGE = 4 * KV_HALF;  // K (2 halves) + V (2 halves)
constexpr int P_BYTES = BM * 128;   // [128 x 64] bf16
constexpr int SOFTMAX_WARPS = 16;
constexpr int THREADS = 64 + SOFTMAX_WARPS * 32;
constexpr int XCH_BYTES = 2 * 4 * BM * 4;  // row exchange [2 buffers][4 parts][128 rows]
constexpr int SMEM = 2 * Q_HALF + KV_STAGES * STAGE + 2 * P_BYTES + XCH_BYTES + 256 + 1024;
constexpr int TMEM_COLS = 512;      // S[b] at column 64b (64 wide), O[b] at 128 + 128b (128 wide)

// bf16(o / l) with the quotient correctly rounded to fp32 first.  y = o * (1/l) (the
// reciprocal correctly rounded) is within 3 fp32 ulps of the rounded quotient q, so bf16(y)
// and bf16(q) agree unless y lies within 3 ulps of a bf16 rounding midpoint (the fp32
// values whose 16 low bits are 0x8000); those, and quotients near the fp32 subnormal
// range, take the IEEE divide.
__device__ __forceinline__ uint16_t bf16_quotient(float o, float l, float rl) {
  float y = o * rl;
  const int d = (int)(__float_as_uint(y) & 0xFFFFu) - 0x8000;
  if ((d > -4 && d < 4) || fabsf(y) < 1e-30f) y = __fdiv_rn(o, l);
  return f2bf(y);
}

struct TcArgs {
  uint16_t* out;
  const int* key_lo;  // per output row: its lowest visible key (several requests in one sequence), or NULL = 0
  // Selected rows (NULL: causal prefill over all T rows).  CTA x computes output row x, the
  // query at position sel[x]: its Q row is row sel[x] of q (q_gather) or row x; the CTA's
  // 128-row Q box starts there and only its first row is kept (a row's arithmetic does not
  // depend on the other rows of its tile, so the bytes equal the causal prefill's row).
  const int64_t* sel;
  int q_gather;
  int T, HQ, HK;
  float scale_log2;  // scale * log2(e)
  float out_inv;     // > 0: e4m3 output, e4m3(clamp(bf16 output * out_inv, +-448)); 0: bf16 output
  // 0: every query row sees every key < T (the vision tower's attention over one image);
  // the tile then visits all key blocks.  1: causal.
  int causal;
  // > 0: the first out_cols columns of each head's output (the rest is zero padding of the
  // head dimension) go to out[row, h * out_cols + c] by plain stores; 0: TMA tile stores
  int out_cols;
  // Rowwise FP8 output (causal prefill, every CTA resident at once): e4m3(bf16 output / s)
  // with s = max(max|row|, 1e-12) / 448 over the row's HQ heads.  headmax[T][HQ] gets each
  // head's maximum of the row, tile_count[T / 128] counts the arrivals per query tile (HQ
  // per launch, never reset: a CTA waits for the next multiple of HQ); qscale[T] gets s.
  float* headmax;
  uint32_t* tile_count;
  float* qscale;
};

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(THREADS, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                        const __grid_constant__ CUtensorMap tmap_v, const __grid_constant__ CUtensorMap tmap_o,
                        const TcArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sq = smem;                          // [2][128 x 128 B]
  uint8_t* skv = sq + 2 * Q_HALF;              // [KV_STAGES][K0 K1 V0 V1]
  uint8_t* sp = skv + KV_STAGES * STAGE;       // P tiles [2]
  float* xch = reinterpret_cast<float*>(sp + 2 * P_BYTES);
  uint64_t* q_full = reinterpret_cast<uint64_t*>(sp + 2 * P_BYTES + XCH_BYTES);
  uint64_t* kv_full = q_full + 1;
  uint64_t* kv_empty = kv_full + KV_STAGES;
  uint64_t* s_full = kv_empty + KV_STAGES;  // [2]
  uint64_t* s_free = s_full + 2;            // [2]
  uint64_t* p_full = s_free + 2;            // [2]
  uint64_t* o_full = p_full + 2;            // [2]
  uint64_t* x_bar = o_full + 2;             // [4]: one per lane quarter, four arrivals
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_bar + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.y, kvh = h / (args.HQ / args.HK);
  const bool rows_mode = args.sel != nullptr;
  // causal prefill: the tile's first query row; selected rows: this row's position
  const int spos = rows_mode ? (int)min(max(args.sel[blockIdx.x], (int64_t)0), (int64_t)(args.T - 1)) : 0;
  const int q0 = rows_mode ? spos : (int)(gridDim.x - 1 - blockIdx.x) * BM;  // heaviest (latest) tiles first
  const int qrow0 = rows_mode ? (args.q_gather ? spos : (int)blockIdx.x) : q0;  // the Q box's first row
  const int kend = !args.causal ? args.T : min(args.T, rows_mode ? spos + 1 : q0 + BM);  // keys this tile sees
  const int nb = (kend + BN - 1) / BN;
  // first key block: the tile's lowest visible key (rows' key_lo are non-decreasing)
  const int lo0 = args.key_lo ? max(args.key_lo[rows_mode ? (int)blockIdx.x : min(q0, args.T - 1)], 0) : 0;
  const int jb0 = min(lo0 / BN, nb);
  const int nit = nb - jb0;                   // key blocks this tile visits

  if (tid == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < KV_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_free[b], SOFTMAX_WARPS);
      mbar_init(&p_full[b], SOFTMAX_WARPS);
      mbar_init(&o_full[b], 1);
    }
    for (int q = 0; q < 4; ++q) mbar_init(&x_bar[q], 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
    tma_prefetch_desc(&tmap_v);
    if (!rows_mode && args.out_cols == 0) tma_prefetch_desc(&tmap_o);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();
  if (tid == 0) pdl_launch();

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_last();
      mbar_arrive_expect_tx(q_full, 2 * Q_HALF);
      tma_load_3d(sq, &tmap_q, q_full, 0, qrow0, h, pol);
      tma_load_3d(sq + Q_HALF, &tmap_q, q_full, 64, qrow0, h, pol);
      int issued = 0;
      for (int j = 0; j < nit && !*abort_flag; ++j, ++issued) {
        const int s = j % KV_STAGES;
        if (j >= KV_STAGES &&
            !mbar_wait_bounded(&kv_empty[s], ((uint32_t)(j / KV_STAGES) & 1u) ^ 1u, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        uint8_t* st = skv + s * STAGE;
        mbar_arrive_expect_tx(&kv_full[s], STAGE);
        const int key = (jb0 + j) * BN;
        tma_load_3d(st, &tmap_k, &kv_full[s], 0, key, kvh, pol);
        tma_load_3d(st + KV_HALF, &tmap_k, &kv_full[s], 64, key, kvh, pol);
        tma_load_3d(st + 2 * KV_HALF, &tmap_v, &kv_full[s], 0, key, kvh, pol);
        tma_load_3d(st + 3 * KV_HALF, &tmap_v, &kv_full[s], 64, key, kvh, pol);
      }
      if (*abort_flag) {  // copies in flight must land before the CTA exits
        volatile int never = 0;
        mbar_wait_bounded(q_full, 0, &never, 200000000ull);
        for (int j = (issued > KV_STAGES ? issued - KV_STAGES : 0); j < issued; ++j)
          mbar_wait_bounded(&kv_full[j % KV_STAGES], (uint32_t)(j / KV_STAGES) & 1u, &never, 200000000ull);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = idesc_bf16(BM, BN);
      constexpr uint32_t idesc_o = idesc_bf16(BM, D) | (1u << 16);  // B (= V) MN-major
      const uint32_t qa = smem_u32(sq);
      // S_j = Q . K_j^T into S[j & 1]
      auto issue_s = [&](int j) -> bool {
        const int st = j % KV_STAGES;
        if (!mbar_wait_bounded(&kv_full[st], (uint32_t)(j / KV_STAGES) & 1u, abort_flag)) return false;
        tc_fence_after();
        const uint32_t kb = smem_u32(skv + st * STAGE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)  // K = head dim: 4 steps of 32 bytes in each half
          umma_f16(tmem + 64 * (j & 1), umma_desc_sw128(qa + (kk >> 2) * Q_HALF + (kk & 3) * 32),
                   umma_desc_sw128(kb + (kk >> 2) * KV_HALF + (kk & 3) * 32), idesc_s, kk > 0 ? 1u : 0u);
        umma_commit(&s_full[j & 1]);
        return true;
      };
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag);
      for (int j = 0; j < 2 && j < nit && ok; ++j) ok = issue_s(j);
      for (int j = 0; j < nit && ok; ++j) {
        const int b = j & 1, st = j % KV_STAGES;
        ok = mbar_wait_bounded(&p_full[b], (uint32_t)(j >> 1) & 1u, abort_flag);
        if (!ok) break;
        tc_fence_after();
        const uint32_t pa = smem_u32(sp + b * P_BYTES), vb = smem_u32(skv + st * STAGE + 2 * KV_HALF);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk)  // K = keys: 16 per step (32 B of P, 2 KB of V)
          umma_f16(tmem + 128 + 128 * b, umma_desc_sw128(pa + kk * 32), umma_desc_sw128_mn(vb + kk * 2048, KV_HALF),
                   idesc_o, kk > 0 ? 1u : 0u);
        umma_commit(&o_full[b]);
        umma_commit(&kv_empty[st]);
        if (j + 2 < nit) {  // S[b] is free once the softmax has read S_j
          ok = mbar_wait_bounded(&s_free[b], (uint32_t)(j >> 1) & 1u, abort_flag);
          if (ok) ok = issue_s(j + 2);
        }
      }
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int part = (warp - 2) >> 2;   // keys [16 part, 16 part + 16), output columns [32 part, 32 part + 32)
    const int r = quarter * 32 + lane;  // this thread's query row in the tile
    // selected rows: every row of the tile masks as row 0; non-causal: as the last row
    const int qpos = !args.causal ? args.T - 1 : rows_mode ? spos : q0 + r;
    const uint32_t lane_addr = (uint32_t)(quarter * 32) << 16;
    float o[D / 4];
#pragma unroll
    for (int i = 0; i < D / 4; ++i) o[i] = 0.f;
    float m = -INFINITY, l = 0.f, alpha_prev = 0.f;
    int xph = 0;  // phases of this quarter's exchange barrier used so far
    // this row's lowest visible key
    const int lo = rows_mode ? lo0 : (args.key_lo && qpos < args.T ? args.key_lo[qpos] : 0);
    // The four parts' values of the row (written to xch[buffer][part][row] by each), in part order.
    auto exchange = [&](float mine, float (&all)[4]) -> bool {
      float* slot = xch + (xph & 1) * 4 * BM;
      slot[part * BM + r] = mine;
      __syncwarp();
      if (lane == 0) mbar_arrive(&x_bar[quarter]);
      const bool got = mbar_wait_bounded(&x_bar[quarter], (uint32_t)xph & 1u, abort_flag);
      ++xph;
#pragma unroll
      for (int p2 = 0; p2 < 4; ++p2) all[p2] = got ? slot[p2 * BM + r] : 0.f;
      return got;
    };
    // o = o * alpha + O_j for this thread's 32 output columns (the fold of block j's P.V)
    auto fold = [&](int j, float alpha) -> bool {
      if (!(mbar_wait_bounded(&o_full[j & 1], (uint32_t)(j >> 1) & 1u, abort_flag) && !*abort_flag)) return false;
      tc_fence_after();
      uint32_t t0[16], t1[16];
      const uint32_t oa = tmem + lane_addr + 128 + 128 * (j & 1) + 32 * part;
      tmem_ld16_async(oa, t0);
      tmem_ld16_async(oa + 16, t1);
      tmem_wait_ld();
      reg_fence(t0);
      reg_fence(t1);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        o[i] = __fmaf_rn(o[i], alpha, __uint_as_float(t0[i]));
        o[16 + i] = __fmaf_rn(o[16 + i], alpha, __uint_as_float(t1[i]));
      }
      tc_fence_before();
      return true;
    };
    bool ok = true;
    for (int j = 0; j < nit && ok; ++j) {
      const int b = j & 1;
      if (!(mbar_wait_bounded(&s_full[b], (uint32_t)(j >> 1) & 1u, abort_flag) && !*abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sr[16];
      tmem_ld16_async(tmem + lane_addr + 64 * b + 16 * part, sr);
      tmem_wait_ld();
      reg_fence(sr);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_free[b]);  // the MMA warp may overwrite S[b]
      // mask (blocks reaching past the tile's first row or past T, or below a row's first
      // visible key) + scale into base 2, in place
      float bmax = -INFINITY;
      const int kb = (jb0 + j) * BN, key0 = kb + 16 * part;
      if ((args.causal && kb + BN - 1 > q0) || kb + BN > args.T || args.key_lo) {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int key = key0 + c;
          const float x =
              (key > qpos || key >= args.T || key < lo) ? -INFINITY : __fmul_rn(__uint_as_float(sr[c]), args.scale_log2);
          sr[c] = __float_as_uint(x);
          bmax = fmaxf(bmax, x);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float x = __fmul_rn(__uint_as_float(sr[c]), args.scale_log2);
          sr[c] = __float_as_uint(x);
          bmax = fmaxf(bmax, x);
        }
      }
      float parts[4];
      if (!exchange(bmax, parts)) {
        *abort_flag = 1;
        ok = false;
        break;
      }
      bmax = fmaxf(fmaxf(parts[0], parts[1]), fmaxf(parts[2], parts[3]));  // the row's maximum over 64 keys
      const float nm = fmaxf(m, bmax);
      const float base = nm == -INFINITY ? 0.f : nm;
      const float alpha = exp2_poly(__fsub_rn(m, base));
      m = nm;
      float psum = 0.f;
      // this part of P_j row r into P[b]: 2 chunks of 16 bytes, 128-byte swizzle.  P[b] was
      // last read by P_{j-2} . V_{j-2}, whose completion the fold of block j-2 waited for.
      uint8_t* prow = sp + b * P_BYTES + r * 128;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p0 = exp2_poly(__fsub_rn(__uint_as_float(sr[8 * c + 2 * e]), base));
          const float p1 = exp2_poly(__fsub_rn(__uint_as_float(sr[8 * c + 2 * e + 1]), base));
          psum = __fadd_rn(psum, __fadd_rn(p0, p1));
          w[e] = (uint32_t)f2bf(p0) | ((uint32_t)f2bf(p1) << 16);
        }
        const int chunk = 2 * part + c;
        *reinterpret_cast<uint4*>(prow + ((chunk ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      l = __fmaf_rn(l, alpha, psum);  // this part's share of the denominator
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
      if (j > 0) ok = fold(j - 1, alpha_prev);  // block j-1's P.V ran while this softmax did
      alpha_prev = alpha;
    }
    if (ok && nit > 0) ok = fold(nit - 1, alpha_prev);
    if (ok) {
      float parts[4];
      ok = exchange(l, parts) && !*abort_flag;
      l = __fadd_rn(__fadd_rn(__fadd_rn(parts[0], parts[1]), parts[2]), parts[3]);  // the four parts, in order
    }
    if (!ok) *abort_flag = 1;
    // Output tile [128 rows x 128 columns] bf16 staged as two 128-byte-swizzled [128 x 64]
    // boxes in the P tiles (every P.V has completed: the last fold waited for it), then TMA
    // stores; rows past T are clipped by the store.
    bool stage = ok && !*abort_flag;
    const bool fp8_out = args.out_inv > 0.f;
    float rscale = 0.f;  // rowwise FP8: this row's scale
    if (args.headmax != nullptr) {
      // Rowwise FP8 output.  o <- the bf16 output values; each head's maximum of the row
      // (over its four parts) goes to headmax; once every head's CTA of the query tile has
      // arrived (a bounded wait: the host launches this only when every CTA of the grid is
      // resident), the maximum over the HQ heads gives the row's scale -- the bytes of
      // ffb_quantize_fp8 (ROWWISE) on the bf16 output.
      const int row = q0 + r, tile = q0 / BM;
      float amax = 0.f;
      if (stage) {
        const float rl = __frcp_rn(l);
#pragma unroll
        for (int i = 0; i < D / 4; ++i) {
          o[i] = bf2f(bf16_quotient(o[i], l, rl));
          amax = fmaxf(amax, fabsf(o[i]));
        }
      }
      float parts[4];
      const bool xok = exchange(amax, parts);
      amax = fmaxf(fmaxf(parts[0], parts[1]), fmaxf(parts[2], parts[3]));
      if (part == 0 && stage && xok && row < args.T) {
        args.headmax[(size_t)row * args.HQ + h] = amax;
        __threadfence();  // visible before this CTA's arrival
      }
      named_barrier(2, SOFTMAX_WARPS * 32);
      volatile int* verdict = reinterpret_cast<volatile int*>(xch);  // the exchange buffers are free now
      if (warp == 2 && lane == 0) {
        int v = 0;
        if (ok && xok && !*abort_flag) {
          const uint32_t old = atomicAdd(args.tile_count + tile, 1u);
          const uint32_t target = (old / (uint32_t)args.HQ + 1u) * (uint32_t)args.HQ;
          const uint64_t t0 = global_timer_ns();
          v = 1;
          uint32_t polls = 0;
          while ((int)(ld_acquire_u32(args.tile_count + tile) - target) < 0) {
            __nanosleep(32);
            if ((++polls & 63u) == 0 && global_timer_ns() - t0 > 2000000000ull) {
              v = 0;
              break;
            }
          }
        }
        *verdict = v;
      }
      named_barrier(2, SOFTMAX_WARPS * 32);
      if (!*verdict) {
        *abort_flag = 1;
        stage = false;
      } else if (row < args.T) {
        // the row's HQ head maxima (L2, bypassing L1), four at a time
        const float* hm = args.headmax + (size_t)row * args.HQ;
        float m = 0.f;
        for (int i = 0; i < args.HQ; i += 4) {
          const float4 f4 = __ldcg(reinterpret_cast<const float4*>(hm + i));
          m = fmaxf(m, fmaxf(fmaxf(f4.x, f4.y), fmaxf(f4.z, f4.w)));
        }
        rscale = __fdiv_rn(fmaxf(m, 1e-12f), 448.f);
        if (h == 0 && part == 0) args.qscale[row] = rscale;
      }
    }
    if (rows_mode) {
      // only the tile's first row is the selected query: its four threads (row 0 of lane
      // quarter 0) store their 32 output columns of output row x with plain stores
      if (stage && r == 0) {
        const float rl = __frcp_rn(l);
        uint16_t* dst = args.out + (size_t)blockIdx.x * args.HQ * D + (size_t)h * D + 32 * part;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = (uint32_t)bf16_quotient(o[8 * c + 2 * e], l, rl) |
                   ((uint32_t)bf16_quotient(o[8 * c + 2 * e + 1], l, rl) << 16);
          *reinterpret_cast<uint4*>(dst + 8 * c) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    } else if (args.out_cols > 0) {
      // direct store: this thread's row, columns [32 part, 32 part + 32) below out_cols (a
      // multiple of 8), 16 bytes at a time
      const int row = q0 + r;
      if (stage && row < args.T) {
        const float rl = __frcp_rn(l);
        uint16_t* dst = args.out + (size_t)row * args.HQ * args.out_cols + (size_t)h * args.out_cols;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int col = 32 * part + 8 * c;
          if (col + 8 > args.out_cols) break;
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = (uint32_t)bf16_quotient(o[8 * c + 2 * e], l, rl) |
                   ((uint32_t)bf16_quotient(o[8 * c + 2 * e + 1], l, rl) << 16);
          *reinterpret_cast<uint4*>(dst + col) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    } else if (stage && args.headmax != nullptr) {
      // one 128-byte-swizzled [128 rows x 128 B] box of e4m3 in P tile 0, as the static path
      uint8_t* orow = sp + r * 128;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t word = 0;
#pragma unroll
          for (int b = 0; b < 4; ++b)
            word |= (uint32_t)f2e4m3(clamp448(__fdiv_rn(o[16 * c + 4 * e + b], rscale))) << (8 * b);
          w[e] = word;
        }
        const int chunk = 2 * part + c;
        *reinterpret_cast<uint4*>(orow + ((chunk ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
    } else if (stage && fp8_out) {
      // the static FP8 quantisation of the o projection's input, applied to the bf16 output:
      // one 128-byte-swizzled [128 rows x 128 B] box in P tile 0, this part's 32 columns
      // as two 16-byte chunks
      const float rl = __frcp_rn(l);
      uint8_t* orow = sp + r * 128;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          uint32_t word = 0;
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const float y = bf2f(bf16_quotient(o[16 * c + 4 * e + b], l, rl));
            word |= (uint32_t)f2e4m3(clamp448(y * args.out_inv)) << (8 * b);
          }
          w[e] = word;
        }
        const int chunk = 2 * part + c;
        *reinterpret_cast<uint4*>(orow + ((chunk ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
    } else if (stage) {
      const float rl = __frcp_rn(l);
      uint8_t* orow = sp + (part >> 1) * P_BYTES + r * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          w[e] = (uint32_t)bf16_quotient(o[8 * c + 2 * e], l, rl) | ((uint32_t)bf16_quotient(o[8 * c + 2 * e + 1], l, rl) << 16);
        const int chunk = 4 * (part & 1) + c;
        *reinterpret_cast<uint4*>(orow + ((chunk ^ (r & 7)) << 4)) = make_uint4(w[0], w[1], w[2], w[3]);
      }
      fence_proxy_async_smem();
    }
    named_barrier(1, SOFTMAX_WARPS * 32);
    if (!rows_mode && args.out_cols == 0 && warp == 2 && lane == 0 && !*abort_flag) {
      if (fp8_out || args.headmax != nullptr) {  // one [128 x 128 B] e4m3 box
        tma_store_2d(&tmap_o, sp, h * D, q0);
      } else {
        tma_store_2d(&tmap_o, sp, h * D, q0);
        tma_store_2d(&tmap_o, sp + P_BYTES, h * D + 64, q0);
      }
      bulk_commit();
      bulk_wait_read<0>();  // the staging tile has been read; the writes complete with the grid
    }
  }

  if (warp == 1 && lane == 0 && *abort_flag) {
    // MMAs already issued must finish before TMEM and shared memory are released
    volatile int never = 0;
    mbar_wait_bounded(&o_full[0], 0, &never, 100000000ull);
    mbar_wait_bounded(&o_full[1], 0, &never, 100000000ull);
  }
  if (tid == 0 && *abort_flag) atomicOr(&ffb_device_error_word, ffb::ERR_ATTN_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace

// Causal self-attention (q, k, v head-major [H, rows, 128] bf16).  sel == NULL: every one
// of the T rows, out [T, HQ*128] (bf16, or e4m3 when out_inv > 0); otherwise the S
// selected rows at positions sel[0..S) (q rows sel[x] of a [HQ, T, 128] q when q_gather,
// else rows x of a [HQ, S, 128] q), out [S, HQ*128] bf16.  key_lo: per output row.
// Called by the host entries of attention.cu after their argument checks.
// causal == 0: every row sees all T keys (sel must be NULL); out_cols > 0: out [T, HQ *
// out_cols] bf16 holds the first out_cols columns of each head (plain stores); rq_sync !=
// NULL: rowwise FP8 output out [T, HQ*128] e4m3 with scales qscale [T], rq_sync the
// [T][HQ] fp32 head maxima followed by [ceil(T/128)] u32 tile counters (the caller checked
// that the grid is resident at once; HQ a multiple of 4).
int ffb_attention_tc(const uint16_t* q, const uint16_t* k, const uint16_t* v, const int64_t* sel, int q_gather,
                     int S, const int* key_lo, void* out, int T, int HQ, int HK, float scale, float out_inv,
                     int causal, int out_cols, void* rq_sync, float* qscale, cudaStream_t stream) {
  CUtensorMap tq, tk, tv, to;
  const uint64_t q_rows = (sel && !q_gather) ? (uint64_t)S : (uint64_t)T;
  int rc = ffb::make_tmap_3d_bf16(&tq, q, D, q_rows, (uint64_t)HQ, 64, BM);
  if (!rc) rc = ffb::make_tmap_3d_bf16(&tk, k, D, (uint64_t)T, (uint64_t)HK, 64, BN);
  if (!rc) rc = ffb::make_tmap_3d_bf16(&tv, v, D, (uint64_t)T, (uint64_t)HK, 64, BN);
  // out [T, HQ*128]: bf16 in [128 rows x 64 columns] boxes, or e4m3 in [128 x 128] boxes
  // (selected rows: plain stores, the map is not used)
  if (sel || out_cols > 0)
    memset(&to, 0, sizeof(to));
  else if (!rc && (out_inv > 0.f || rq_sync))
    rc = ffb::make_tmap_2d(&to, out, (uint64_t)T, (uint64_t)HQ * D, (uint64_t)HQ * D, BM, 128, 1);
  else if (!rc)
    rc = ffb::make_tmap_2d(&to, out, (uint64_t)T, (uint64_t)HQ * D, (uint64_t)HQ * D * 2, BM, 64, 2);
  if (rc) return rc;
  cudaError_t e = ffb::set_smem_attr(reinterpret_cast<const void*>(attention_tc_kernel), SMEM);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_attention: %s", cudaGetErrorString(e));
  TcArgs a = {static_cast<uint16_t*>(out), key_lo, sel, q_gather, T, HQ, HK, scale * 1.4426950408889634f, out_inv,
              causal, out_cols, static_cast<float*>(rq_sync),
              rq_sync ? reinterpret_cast<uint32_t*>(static_cast<float*>(rq_sync) + (size_t)T * HQ) : nullptr, qscale};
  const dim3 grid(sel ? S : (T + BM - 1) / BM, HQ);
  e = ffb::launch(attention_tc_kernel, grid, dim3(THREADS), SMEM, stream, tq, tk, tv, to, a);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_attention: %s", cudaGetErrorString(e));
  return FFB_OK;
}
