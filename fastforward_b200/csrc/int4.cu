// W4A16 path: symmetric int4 group-128 weight packing (the GEMM is gemm_w4a16.cu).
//
// Packing (set-up): per group of 128 along K, s = bf16(max|W|/7) (floored at 1e-8),
// q = clamp(rne(W/s), -8, 7), two nibbles per byte (low nibble = even k).
// Replaces the packing in _family/night_runtime.py:15-26 (`Int4.__init__`, asymmetric
// group 32 there) with the symmetric group-128 scheme the W4A16 configuration uses.
#include "common.cuh"
#include "pdl.cuh"

namespace {

// One warp per (row, group): lane l handles elements 4l..4l+3 of the group.
__global__ void __launch_bounds__(256) pack_int4_kernel(const uint16_t* __restrict__ w, uint8_t* __restrict__ packed,
                                                        uint16_t* __restrict__ scales, int N, int K) {
  pdl_wait();
  pdl_launch();
  const int lane = threadIdx.x & 31;
  const long long item = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int groups = K / 128;
  if (item >= (long long)N * groups) return;
  const int n = (int)(item / groups), gi = (int)(item % groups);
  const uint16_t* src = w + (size_t)n * K + gi * 128 + lane * 4;
  float x[4];
  float amax = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    x[e] = bf2f(src[e]);
    amax = fmaxf(amax, fabsf(x[e]));
  }
  amax = warp_max(amax);
  const float s = round_bf(__fdiv_rn(fmaxf(amax, 1e-8f), 7.f));
  if (lane == 0) scales[(size_t)n * groups + gi] = f2bf(s);
  uint32_t nib[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float q = rintf(__fdiv_rn(x[e], s));
    q = fminf(7.f, fmaxf(-8.f, q));
    nib[e] = (uint32_t)((int)q & 0xF);
  }
  uint8_t* dst = packed + (size_t)n * (K / 2) + gi * 64 + lane * 2;
  dst[0] = (uint8_t)(nib[0] | (nib[1] << 4));
  dst[1] = (uint8_t)(nib[2] | (nib[3] << 4));
}

}  // namespace

extern "C" int ffb_pack_int4(const uint16_t* w, uint8_t* packed, uint16_t* scales, int N, int K, void* stream) {
  FFB_REQUIRE(w && packed && scales, "ffb_pack_int4: NULL pointer");
  FFB_REQUIRE(N > 0 && K > 0 && K % 128 == 0, "ffb_pack_int4: K=%d must be a multiple of 128", K);
  const long long items = (long long)N * (K / 128);
  cudaError_t e = ffb::launch(pack_int4_kernel, dim3((unsigned)((items + 7) / 8)), dim3(256), 0, (cudaStream_t)stream,
                              w, packed, scales, N, K);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_pack_int4: %s", cudaGetErrorString(e));
  return FFB_OK;
}
