// Raw RGB canvas -> vision patch rows (the input packing in front of the vision tower).
//
// Reference: `pack_rgb` (`_legacy/sub10_runtime.py:21-29`, square canvases) and
// `pack_rectangle` (`_family/depth_runtime.py:18-25`, any canvas of 32-pixel multiples).
// The canvas [height, width, 3] u8 (HWC) becomes [(height/16)(width/16), 1536] bf16: one
// row per 16x16 patch, patches ordered by 2x2 merge group (group-row-major; inside a group
// top-left, top-right, bottom-left, bottom-right), each row = 3 channels x 2 temporal
// copies x 16 x 16 pixels, value (u8 - 127.5) / 127.5 rounded to bf16.
//
// HBM-bound byte work (3 bytes read, 12 bytes written per pixel).  One warp per patch
// row, one thread per half pixel row: 24 contiguous input bytes (8 RGB pixels, three
// 8-byte loads when the canvas is 8-byte aligned) and six 16-byte stores, which the warp
// issues as six fully coalesced 512-byte runs (one per channel and temporal copy).
#include "common.cuh"
#include "pdl.cuh"

namespace {
constexpr int PATCH = 16;
constexpr int PATCH_ROW = 3 * 2 * PATCH * PATCH;  // 1536 values per patch row

// (u8 - 127.5) / 127.5 in fp32, rounded to bf16 (nearest even, the reference's store into
// a bf16 tensor).  Computed as (u8 - 127.5) * fp32(2/255): byte k of `word` becomes the
// mantissa of 2^23 + u8 (one byte permute), both subtractions are exact, and the product
// is within one fp32 ulp of the IEEE quotient.  For every byte value the bf16 of the
// product equals the bf16 of the IEEE quotient (no quotient lies near a bf16 rounding
// boundary); the host test suite checks all 256 exhaustively.
constexpr float TWO_OVER_255 = 0x1.010102p-7f;  // 2/255 correctly rounded to fp32

__device__ __forceinline__ float byte_value(uint32_t word, int k) {
  const float m = __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7650u | (uint32_t)k));
  return __fmul_rn(__fsub_rn(__fsub_rn(m, 8388608.0f), 127.5f), TWO_OVER_255);
}

__device__ __forceinline__ uint32_t bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <bool ALIGNED>
__global__ void __launch_bounds__(256) pack_rgb_kernel(const uint8_t* __restrict__ rgb,
                                                       uint16_t* __restrict__ pixels, int height, int width,
                                                       int patches, int n_threads) {
  pdl_wait();
  pdl_launch();
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n_threads) return;
  // one warp per patch row: lane = (pixel row y0, half xh of the 16-pixel row)
  const int pg = g >> 5, y0 = (g >> 1) & 15, xh = g & 1;
  const int img = pg / patches, p = pg - img * patches;
  const int groups_w = width / 32;  // 2x2 merge groups per canvas row
  const int grp = p >> 2, my = (p >> 1) & 1, mx = p & 1;
  const int y = (grp / groups_w) * 32 + my * 16 + y0;
  const int x = (grp % groups_w) * 32 + mx * 16 + xh * 8;
  const uint8_t* src = rgb + (((size_t)img * height + y) * width + x) * 3;
  uint32_t w[6];  // 24 bytes: pixel j channel c is byte 3j + c
  if constexpr (ALIGNED) {
    const uint2* s2 = reinterpret_cast<const uint2*>(src);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const uint2 v = __ldg(s2 + i);
      w[2 * i] = v.x;
      w[2 * i + 1] = v.y;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 6; ++i)
      w[i] = (uint32_t)src[4 * i] | (uint32_t)src[4 * i + 1] << 8 | (uint32_t)src[4 * i + 2] << 16 |
             (uint32_t)src[4 * i + 3] << 24;
  }
  // the warp's 32 lanes store 32 consecutive 16-byte chunks: 512 contiguous bytes per store
  uint16_t* row = pixels + (size_t)pg * PATCH_ROW + y0 * PATCH + xh * 8;
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b0 = 3 * (2 * j) + c, b1 = 3 * (2 * j + 1) + c;
      o[j] = bf16x2(byte_value(w[b0 >> 2], b0 & 3), byte_value(w[b1 >> 2], b1 & 3));
    }
    const uint4 v = make_uint4(o[0], o[1], o[2], o[3]);
#pragma unroll
    for (int t = 0; t < 2; ++t)  // the two temporal copies of the still image
      *reinterpret_cast<uint4*>(row + c * 512 + t * 256) = v;
  }
}
}  // namespace

extern "C" int ffb_pack_rgb_batch(const uint8_t* rgb, uint16_t* pixels, int n, int height, int width,
                                  void* stream) {
  FFB_REQUIRE(rgb && pixels, "ffb_pack_rgb: NULL pointer");
  FFB_REQUIRE(n >= 1, "ffb_pack_rgb_batch: n=%d canvases", n);
  FFB_REQUIRE(height > 0 && width > 0 && height % 32 == 0 && width % 32 == 0,
              "ffb_pack_rgb: canvas %dx%d must be positive multiples of 32 (2x2 groups of 16-pixel patches)", height,
              width);
  FFB_REQUIRE((long long)n * height * width <= (1ll << 30), "ffb_pack_rgb: %d canvases of %dx%d exceed 2^30 pixels",
              n, height, width);
  FFB_REQUIRE(ffb::aligned(pixels, 16), "ffb_pack_rgb: pixels must be 16-byte aligned");
  const int patches = (height / PATCH) * (width / PATCH);
  const int threads = n * patches * 32;  // <= 2^27
  const dim3 grid((threads + 255) / 256), block(256);
  cudaError_t e;
  if (ffb::aligned(rgb, 8))
    e = ffb::launch(pack_rgb_kernel<true>, grid, block, 0, (cudaStream_t)stream, rgb, pixels, height, width, patches,
                    threads);
  else
    e = ffb::launch(pack_rgb_kernel<false>, grid, block, 0, (cudaStream_t)stream, rgb, pixels, height, width, patches,
                    threads);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_pack_rgb: %s", cudaGetErrorString(e));
  return FFB_OK;
}

extern "C" int ffb_pack_rgb(const uint8_t* rgb, uint16_t* pixels, int height, int width, void* stream) {
  return ffb_pack_rgb_batch(rgb, pixels, 1, height, width, stream);
}
