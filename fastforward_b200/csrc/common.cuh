// Shared helpers of libffb200: error reporting, bf16/fp8 conversions, and the sm_100a
// PTX wrappers (mbarrier, TMA, tcgen05) the tensor-core kernels are written with.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include <stdio.h>
#include <string>

#include "../../include/ffb200.h"

namespace ffb {

// ------------------------------------------------------------------ host error plumbing
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_launch(const char* what);
// Raises `fn`'s dynamic shared-memory limit to `bytes` on the current device, once per
// (function, device); thread-safe.
cudaError_t set_smem_attr(const void* fn, int bytes);
// Streaming multiprocessors of the current device.
int sm_count();

// The weight-stationary FP8 GEMM (gemm_fp8_stream.cu): weights on the MMA's M side, tokens
// on N, one (weight tile, token range, K range) item per CTA.  `ctas` is its CTA count for
// this M x N x K, epilogue (FFB_EPI_BF16, FFB_EPI_F32_PARTIAL, FFB_EPI_SWIGLU, 100 = qkv +
// QK-norm + RoPE, 101 = SwiGLU + static FP8 output) and K split, or 0 when it does not
// apply; `stream_gemm` runs it (the caller has checked the arguments; rope_side points to
// the qkv epilogue's argument block).
int stream_gemm_ctas(int M, int N, int K, int epilogue, int splits);
bool stream_gemm_preferred(int M, int N, int K, int epilogue);
int stream_gemm(const uint8_t* a8, const float* a_scale, int a_per_row, const uint8_t* w8, const float* w_scale,
                int w_per_col, int epilogue, void* out, int splits, float out_inv, const void* rope_side, int M, int N,
                int K, cudaStream_t stream);

#define FFB_REQUIRE(cond, ...)                                   \
  do {                                                           \
    if (!(cond)) return ::ffb::fail(FFB_EINVAL, __VA_ARGS__);    \
  } while (0)

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Bits of the per-device error word (set by kernels whose bounded wait gave up).
enum : uint32_t {
  ERR_GEMM_TIMEOUT = 1u << 0,
  ERR_W4_TIMEOUT = 1u << 1,
  ERR_ATTN_TIMEOUT = 1u << 2,
  ERR_GRID_SYNC_TIMEOUT = 1u << 3,
  ERR_PEER_TIMEOUT = 1u << 4,
};

// Fills ffb_silu_table on this device once (stream-ordered, before the caller's next
// launch); inside a stream capture the fill is captured as well and the table is marked
// filled only by an uncaptured call.
int ensure_silu_table(cudaStream_t stream);

}  // namespace ffb

// One error word per device that loads the library.
extern __device__ uint32_t ffb_device_error_word;

// ------------------------------------------------------------------ numeric helpers
__device__ __forceinline__ float bf2f(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }
__device__ __forceinline__ uint16_t f2bf(float f) {  // round to nearest even
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float round_bf(float f) { return bf2f(f2bf(f)); }

// SiLU of a bf16 value as the reference rounds it, bf16(g / (1 + exp(-g))) with an IEEE
// divide (_legacy/search_kernels.py:14).
__device__ __forceinline__ float silu_bf16(float g) { return round_bf(__fdiv_rn(g, 1.f + expf(-g))); }

// silu_bf16 of every bf16 value, indexed by its bits (filled by ffb::ensure_silu_table):
// the SwiGLU epilogues look the activation up instead of evaluating exp and a division.
extern __device__ uint16_t ffb_silu_table[65536];
__device__ __forceinline__ float silu_lookup(float g_bf16) {
  return bf2f(__ldg(&ffb_silu_table[__float_as_uint(g_bf16) >> 16]));
}
// fp32 -> e4m3 with round-to-nearest-even; the callers clamp to +-448 first, so the
// saturating conversion never sees an out-of-range value.
__device__ __forceinline__ uint8_t f2e4m3(float f) {
  return (uint8_t)__nv_cvt_float_to_fp8(f, __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ float clamp448(float v) { return fminf(448.f, fmaxf(-448.f, v)); }

// e4m3 byte of clamp(x / s, +-448) with x / s correctly rounded, for the rowwise
// quantisers: s = max(a, 1e-12) / 448 with a the row's largest |x|, r = 1 / s correctly
// rounded (__frcp_rn, once per row).  Instead of an IEEE divide per element (a multi-
// instruction sequence that dominated the quantisers' time): q0 = x r, one fused-multiply-
// add correction q = q0 + (x - q0 s) r, and x's sign bit set on q (so that -0 / s stays -0).
// For every bf16 x with |x| <= a and every non-negative finite bf16 a -- the whole domain of
// these callers -- the byte equals the divide's; checked exhaustively over all
// 1,065,402,240 (a, x) pairs on the CPU (tests/test_rowdiv_exhaustive.py).  The fp32
// quotients themselves differ only below 6e-20, where both round to a zero byte.  A
// non-finite s (a row holding an infinity) takes the divide.
__device__ __forceinline__ uint32_t e4m3_quotient(float x, float s, float r) {
  float q;
  if (isfinite(s)) {
    const float q0 = __fmul_rn(x, r);
    q = __fmaf_rn(__fmaf_rn(-q0, s, x), r, q0);
    q = __uint_as_float(__float_as_uint(q) | (__float_as_uint(x) & 0x80000000u));
  } else {
    q = __fdiv_rn(x, s);
  }
  return f2e4m3(clamp448(q));
}

// exp2_poly: 2^x = 2^n * 2^f with n = rint(x) and f = x - n in [-1/2, 1/2] (exact); 2^f
// is the degree-7 Taylor polynomial of e^(f ln 2) (coefficients (ln 2)^k / k! rounded to
// fp32) in Horner form with fused multiply-adds, and 2^n is added to the exponent field.
// Results below 2^-125 (and x = -inf) are 0; x must stay below 128.  Within a few ulps of
// 2^x; every operation is an IEEE-rounded one, so a CPU with fmaf reproduces it.
__device__ __forceinline__ float exp2_poly(float x) {
  if (!(x >= -125.f)) return 0.f;
  const float n = rintf(x);
  const float f = __fsub_rn(x, n);
  float p = 1.52527338040598403e-05f;
  p = __fmaf_rn(p, f, 0.000154035303933816099f);
  p = __fmaf_rn(p, f, 0.00133335581464284434f);
  p = __fmaf_rn(p, f, 0.00961812910762847717f);
  p = __fmaf_rn(p, f, 0.0555041086648215800f);
  p = __fmaf_rn(p, f, 0.240226506959100712f);
  p = __fmaf_rn(p, f, 0.693147180559945309f);
  p = __fmaf_rn(p, f, 1.f);
  return __int_as_float(__float_as_int(p) + ((int)n << 23));
}



__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
// 1 / sqrt(ss/n + eps) from an exact (float64) sum of squares: the sum rounded to fp32,
// IEEE divide, IEEE square root, IEEE reciprocal -- reproducible on any IEEE machine and
// independent of the reduction order.
__device__ __forceinline__ float inv_rms_from_ss(double ss, int n, float eps) {
  const float var = __fdiv_rn((float)ss, (float)n);
  return __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(var, eps)));
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ------------------------------------------------------------------ PTX: shared memory, mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase.  Gives up after ~`limit_ns` of wall time (checked
// every 256 polls) or 2^26 polls, or as soon as *abort is set by another role of the CTA.
// Returns false when it gave up; the caller then records the error and unwinds.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort,
                                                  uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t i = 1; i < (1u << 26); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > limit_ns) return false;
    }
  }
  return false;
}

// ------------------------------------------------------------------ grid-wide barrier
__device__ __forceinline__ uint64_t ld_acquire_gpu_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t atom_add_acq_rel_gpu(uint64_t* p, uint64_t v) {
  uint64_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(v) : "memory");
  return old;
}
// Orders this thread's earlier generic-proxy accesses to global memory before its later
// async-proxy (TMA) accesses.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Barrier over every CTA of the grid, for kernels whose CTAs are all resident at once
// (one per SM, grid <= SMs: the host checks the occupancy).  One 64-bit word: the high
// half is the generation, the low half counts arrivals.  Each CTA's thread 0 arrives with
// an acq_rel atomic add (releasing the CTA's writes, ordered before it by __syncthreads);
// the last arrival adds 2^32 - G, which clears the count and advances the generation in
// one atomic, so the word needs no reset between launches (launches that use the same
// word must not overlap: one word per stream).  The others poll the word with acquire
// loads.  Thread 0 gives up after `limit_ns`; the result (the same in every thread) is
// false then.
__device__ __forceinline__ bool grid_barrier(uint64_t* bar, int* flag_smem, uint64_t limit_ns = 2000000000ull) {
  __syncthreads();
  if (threadIdx.x == 0) {
    int ok = 1;
    const uint64_t old = atom_add_acq_rel_gpu(bar, 1ull);
    const uint32_t gen = (uint32_t)(old >> 32);
    if ((uint32_t)old + 1u == gridDim.x) {
      atom_add_acq_rel_gpu(bar, (1ull << 32) - (uint64_t)gridDim.x);
    } else {
      const uint64_t t0 = global_timer_ns();
      uint32_t polls = 0;
      while ((uint32_t)(ld_acquire_gpu_u64(bar) >> 32) == gen) {
        if ((++polls & 63u) == 0 && global_timer_ns() - t0 > limit_ns) {
          ok = 0;
          break;
        }
      }
    }
    *flag_smem = ok;
  }
  __syncthreads();
  return *flag_smem != 0;
}

// ------------------------------------------------------------------ PTX: TMA
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(policy)
      : "memory");
}
// Shared -> global tile store (bulk async group); rows/columns outside the tensor are
// clipped by the hardware.  x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
// Barrier over `count` threads (whole warps) of the CTA on hardware barrier `id` (1..15).
__device__ __forceinline__ void named_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {  // the last N groups may still be pending
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's prior shared-memory writes before later async-proxy (TMA) reads.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ------------------------------------------------------------------ PTX: thread-block clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The address of this CTA's shared-memory location `p` in cluster CTA `rank`'s window.
__device__ __forceinline__ uint32_t cluster_map(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
  return out;
}
__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
// Cluster-wide barrier: every thread of every CTA of the cluster arrives (release) and
// waits (acquire), so shared-memory writes before it are visible to every CTA after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// ------------------------------------------------------------------ PTX: tcgen05 / TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {  // whole warp
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, e4m3 x e4m3 -> f32.  One thread issues.
__device__ __forceinline__ void umma_f8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// bf16 x bf16 -> f32 (both operands the same type, as kind::f16 requires).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Asynchronous TMEM loads (no wait): the registers are valid only after tmem_wait_ld()
// followed by reg_fence() on them, which ties every later use to the wait.
__device__ __forceinline__ void tmem_ld8_async(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16_async(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
template <int N>
__device__ __forceinline__ void reg_fence(uint32_t (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(r[i]));
}
// Requests the 128-byte line holding p into L1 (a hint: no fault, no result).
__device__ __forceinline__ void prefetch_l1(const void* p) { asm volatile("prefetch.global.L1 [%0];" ::"l"(p)); }
// Eight consecutive fp32 values (16-byte aligned) through the read-only path.
__device__ __forceinline__ void ldg8(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// 32 lanes x 32 consecutive fp32 columns: thread i of the warp gets lane (taddr.lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 32 lanes x 16 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr));
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// UMMA shared-memory matrix descriptor: K-major operand staged by TMA with 128-byte
// swizzle (8-row x 128-byte atoms, atoms packed every 1024 bytes).  The tile base must be
// 1024-byte aligned; stepping K inside the atom adds the byte offset to the start address.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);  // start address
  d |= (uint64_t)1 << 16;                        // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;              // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;                        // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                        // layout: 128-byte swizzle
  return d;
}

// Instruction descriptors (dense, f32 accumulate, both operands K-major).
// UMMA shared-memory descriptor for an MN-major operand staged with the 128-byte swizzle:
// 64 MN elements (128 bytes) per line, 8 K lines per 1024-byte atom (SBO = 1024 between
// K groups of 8), MN chunks of 64 elements `lbo_bytes` apart.
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
__host__ __device__ constexpr uint32_t idesc_e4m3(int M, int N) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------ host: TMA descriptors
namespace ffb {
// 2-D K-major tile map: rows x cols (cols contiguous, `row_bytes` apart), box box_rows x
// box_cols elements of `elem_bytes`, 128-byte swizzle, zero fill out of bounds.
int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_bytes,
                 uint32_t box_rows, uint32_t box_cols, int elem_bytes);
// 3-D bf16 load map [depth][rows][inner] (contiguous), box box_inner (= 64, 128 bytes) x
// box_rows x 1, 128-byte swizzle; rows past `rows` of a depth slice are zero filled.
int make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t depth,
                      uint32_t box_inner, uint32_t box_rows);
// 2-D byte map without swizzle: rows x cols bytes, box box_rows x box_cols (box_cols a
// multiple of 16), zero fill out of bounds; the tile lands row after row in shared memory.
int make_tmap_2d_bytes(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_bytes,
                       uint32_t box_rows, uint32_t box_cols);
// 3-D byte map without swizzle: [depth][rows][inner bytes] (row and plane pitches in
// bytes), box {box_inner bytes (a multiple of 16), box_rows, 1}; out-of-range rows of a
// plane are clipped (stores) or zero filled (loads).
int make_tmap_3d_bytes(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t depth,
                       uint64_t row_bytes, uint64_t depth_bytes, uint32_t box_inner, uint32_t box_rows);
// 3-D store map [depth][rows][inner] (bf16 or fp32), box {64 bytes, box_rows, 1}, 64-byte
// swizzle: the staging tile in shared memory holds row r's 16-byte chunk c at
// r*64 + ((c ^ ((r >> 1) & 3)) << 4), in a buffer aligned to 512 bytes.
int make_tmap_out(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t rows,
                  uint64_t depth, uint64_t row_bytes, uint64_t depth_bytes, uint32_t box_inner, uint32_t box_rows);
}  // namespace ffb
