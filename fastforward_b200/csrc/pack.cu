// Raw RGB canvas -> vision patch rows (the input packing in front of the vision tower).
//
// Reference: `pack_rgb` (`_legacy/sub10_runtime.py:21-29`, square canvases) and
// `pack_rectangle` (`_family/depth_runtime.py:18-25`, any canvas of 32-pixel multiples).
// The canvas [height, width, 3] u8 (HWC) becomes [(height/16)(width/16), 1536] bf16: one
// row per 16x16 patch, patches ordered by 2x2 merge group (group-row-major; inside a group
// top-left, top-right, bottom-left, bottom-right), each row = 3 channels x 2 temporal
// copies x 16 x 16 pixels, value (u8 - 127.5) / 127.5 rounded to bf16.
//
// HBM-bound byte work (3 bytes read, 12 bytes written per pixel).  One thread per
// (patch, pixel row): 48 contiguous input bytes (16 RGB pixels, three 16-byte loads when
// the canvas is 16-byte aligned) and six 32-byte runs of output, so a warp writes two
// patches' rows as contiguous 512-byte runs.
#include "common.cuh"
#include "pdl.cuh"

namespace {
constexpr int PATCH = 16;
constexpr int PATCH_ROW = 3 * 2 * PATCH * PATCH;  // 1536 values per patch row

// (u8 - 127.5) / 127.5 in fp32 (IEEE division, as the reference's fp32 `/`), bf16 bits
// rounded to nearest even (the reference's store into a bf16 tensor).  The u8 operand
// makes the subtraction exact; no quotient lies within a few fp32 ulps of a bf16 rounding
// boundary, so the bf16 result does not depend on the division's last bit.
__device__ __forceinline__ uint32_t pixel_bf16(uint32_t raw) {
  const float v = __fdiv_rn(static_cast<float>(raw) - 127.5f, 127.5f);
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

template <bool ALIGNED>
__global__ void __launch_bounds__(256) pack_rgb_kernel(const uint8_t* __restrict__ rgb,
                                                       uint16_t* __restrict__ pixels, int height, int width,
                                                       int patches, int n_threads) {
  pdl_wait();
  pdl_launch();
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  if (g >= n_threads) return;
  const int pg = g >> 4, y0 = g & 15;       // patch row over all canvases, pixel row in it
  const int img = pg / patches, p = pg - img * patches;
  const int groups_w = width / 32;           // 2x2 merge groups per canvas row
  const int grp = p >> 2, my = (p >> 1) & 1, mx = p & 1;
  const int y = (grp / groups_w) * 32 + my * 16 + y0;
  const int x = (grp % groups_w) * 32 + mx * 16;
  const uint8_t* src = rgb + (((size_t)img * height + y) * width + x) * 3;
  uint32_t w[12];  // 48 bytes: pixel j channel c is byte 3j + c
  if constexpr (ALIGNED) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int i = 0; i < 3; ++i) {
      const uint4 v = __ldg(s4 + i);
      w[4 * i] = v.x;
      w[4 * i + 1] = v.y;
      w[4 * i + 2] = v.z;
      w[4 * i + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 12; ++i)
      w[i] = (uint32_t)src[4 * i] | (uint32_t)src[4 * i + 1] << 8 | (uint32_t)src[4 * i + 2] << 16 |
             (uint32_t)src[4 * i + 3] << 24;
  }
  uint16_t* row = pixels + (size_t)pg * PATCH_ROW + y0 * PATCH;
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    uint32_t o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int b0 = 3 * (2 * j) + c, b1 = 3 * (2 * j + 1) + c;
      const uint32_t r0 = (w[b0 >> 2] >> ((b0 & 3) * 8)) & 0xFFu;
      const uint32_t r1 = (w[b1 >> 2] >> ((b1 & 3) * 8)) & 0xFFu;
      o[j] = pixel_bf16(r0) | pixel_bf16(r1) << 16;
    }
    const uint4 lo = make_uint4(o[0], o[1], o[2], o[3]), hi = make_uint4(o[4], o[5], o[6], o[7]);
#pragma unroll
    for (int t = 0; t < 2; ++t) {  // the two temporal copies of the still image
      uint4* d = reinterpret_cast<uint4*>(row + c * 512 + t * 256);
      d[0] = lo;
      d[1] = hi;
    }
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
  const int threads = n * patches * PATCH;  // <= 2^26
  const dim3 grid((threads + 255) / 256), block(256);
  cudaError_t e;
  if (ffb::aligned(rgb, 16))
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
