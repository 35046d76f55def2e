// Library-wide host plumbing: thread-local error messages, the per-device error word,
// and TMA descriptor encoding through the driver entry point (no link against libcuda).
#include "common.cuh"
#include "pdl.cuh"

#include <stdarg.h>
#include <string.h>
#include <atomic>
#include <mutex>

__device__ uint32_t ffb_device_error_word = 0;
__device__ uint16_t ffb_silu_table[65536];

namespace {

__global__ void silu_table_kernel() {
  pdl_wait();  // keeps the programmatic-launch chain transitive for the kernels after it
  pdl_launch();
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  ffb_silu_table[i] = f2bf(silu_bf16(bf2f((uint16_t)i)));
}

std::atomic<int> g_silu_filled[64];

}  // namespace

namespace ffb {

int g_use_pdl = 1;

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return code;
}

// (function, device) pairs whose dynamic shared-memory limit is already raised.  The
// attribute is per function and per device, so a process that drives several devices
// sets it once on each; the table is guarded by a mutex (host threads may launch
// concurrently).
namespace {
constexpr int kAttrSlots = 256;
struct AttrSlot {
  const void* fn;
  int dev;
  int bytes;
};
AttrSlot g_attr[kAttrSlots];
int g_attr_n = 0;
std::mutex g_attr_mu;
}  // namespace

cudaError_t set_smem_attr(const void* fn, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_attr_mu);
  for (int i = 0; i < g_attr_n; ++i)
    if (g_attr[i].fn == fn && g_attr[i].dev == dev && g_attr[i].bytes >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  if (g_attr_n < kAttrSlots) g_attr[g_attr_n++] = AttrSlot{fn, dev, bytes};
  return cudaSuccess;
}

int sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) return 148;
  return sms;
}

int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(FFB_ECUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return FFB_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int make_tmap_2d(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_bytes,
                 uint32_t box_rows, uint32_t box_cols, int elem_bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(FFB_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  if (!aligned(base, 16)) return fail(FFB_EINVAL, "TMA base address must be 16-byte aligned");
  if (row_bytes % 16 != 0) return fail(FFB_EINVAL, "TMA row pitch (%llu bytes) must be a multiple of 16",
                                       (unsigned long long)row_bytes);
  if ((uint64_t)box_cols * elem_bytes != 128)
    return fail(FFB_EINVAL, "TMA box inner extent must be 128 bytes for the 128-byte swizzle");
  CUtensorMapDataType dt = elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FFB_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return FFB_OK;
}

int make_tmap_3d_bf16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t depth,
                      uint32_t box_inner, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(FFB_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  if (!aligned(base, 16)) return fail(FFB_EINVAL, "TMA base address must be 16-byte aligned");
  if ((inner * 2) % 16 != 0) return fail(FFB_EINVAL, "TMA row pitch must be a multiple of 16 bytes");
  if (box_inner * 2 != 128) return fail(FFB_EINVAL, "TMA box inner extent must be 128 bytes for the 128-byte swizzle");
  cuuint64_t dims[3] = {inner, rows, depth};
  cuuint64_t strides[2] = {inner * 2, inner * 2 * rows};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FFB_ECUDA, "cuTensorMapEncodeTiled (3d) failed (%d)", (int)r);
  return FFB_OK;
}

int make_tmap_2d_bytes(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t row_bytes,
                       uint32_t box_rows, uint32_t box_cols) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(FFB_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  if (!aligned(base, 16)) return fail(FFB_EINVAL, "TMA base address must be 16-byte aligned");
  if (row_bytes % 16 != 0) return fail(FFB_EINVAL, "TMA row pitch (%llu bytes) must be a multiple of 16",
                                       (unsigned long long)row_bytes);
  if (box_cols % 16 != 0 || box_cols > 256 || box_rows > 256)
    return fail(FFB_EINVAL, "TMA byte box %u x %u: inner extent a multiple of 16, both <= 256", box_cols, box_rows);
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FFB_ECUDA, "cuTensorMapEncodeTiled (bytes) failed (%d)", (int)r);
  return FFB_OK;
}

int make_tmap_3d_bytes(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t depth,
                       uint64_t row_bytes, uint64_t depth_bytes, uint32_t box_inner, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(FFB_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  if (!aligned(base, 16)) return fail(FFB_EINVAL, "TMA base address must be 16-byte aligned");
  if (row_bytes % 16 != 0 || depth_bytes % 16 != 0)
    return fail(FFB_EINVAL, "TMA strides (%llu, %llu bytes) must be multiples of 16", (unsigned long long)row_bytes,
                (unsigned long long)depth_bytes);
  if (box_inner % 16 != 0 || box_inner > 256 || box_rows > 256)
    return fail(FFB_EINVAL, "TMA byte box %u x %u: inner extent a multiple of 16, both <= 256", box_inner, box_rows);
  cuuint64_t dims[3] = {inner, rows, depth};
  cuuint64_t strides[2] = {row_bytes, depth_bytes};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FFB_ECUDA, "cuTensorMapEncodeTiled (3-D bytes) failed (%d)", (int)r);
  return FFB_OK;
}

int make_tmap_out(CUtensorMap* map, const void* base, int elem_bytes, uint64_t inner, uint64_t rows,
                  uint64_t depth, uint64_t row_bytes, uint64_t depth_bytes, uint32_t box_inner, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(FFB_ECUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
  if (!aligned(base, 16)) return fail(FFB_EINVAL, "TMA base address must be 16-byte aligned");
  if (row_bytes % 16 != 0 || depth_bytes % 16 != 0)
    return fail(FFB_EINVAL, "TMA strides (%llu, %llu bytes) must be multiples of 16", (unsigned long long)row_bytes,
                (unsigned long long)depth_bytes);
  // 16/32-bit elements: 64-byte boxes with the 64-byte swizzle; bytes: 32-byte unswizzled boxes
  if ((uint64_t)box_inner * elem_bytes != (elem_bytes == 1 ? 32u : 64u))
    return fail(FFB_EINVAL, "store box must be %d bytes wide", elem_bytes == 1 ? 32 : 64);
  const CUtensorMapDataType dt = elem_bytes == 4   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : elem_bytes == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  cuuint64_t dims[3] = {inner, rows, depth};
  cuuint64_t strides[2] = {row_bytes, depth_bytes};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  elem_bytes == 1 ? CU_TENSOR_MAP_SWIZZLE_NONE : CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FFB_ECUDA, "cuTensorMapEncodeTiled (store) failed (%d)", (int)r);
  return FFB_OK;
}

int ensure_silu_table(cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(FFB_ECUDA, "silu table: %s", cudaGetErrorString(e));
  if (dev >= 0 && dev < 64 && g_silu_filled[dev].load(std::memory_order_acquire)) return FFB_OK;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(stream, &cap);
  if (e == cudaSuccess) e = launch(silu_table_kernel, dim3(65536 / 256), dim3(256), 0, stream);
  if (e != cudaSuccess) return fail(FFB_ECUDA, "silu table: %s", cudaGetErrorString(e));
  if (cap == cudaStreamCaptureStatusNone && dev >= 0 && dev < 64) g_silu_filled[dev].store(1, std::memory_order_release);
  return FFB_OK;
}

}  // namespace ffb

extern "C" {

const char* ffb_version(void) { return "ffb200 0.1.0 sm_100a"; }

int ffb_set_pdl(int enable) {
  const int old = ffb::g_use_pdl;
  ffb::g_use_pdl = enable ? 1 : 0;
  return old;
}

int ffb_last_error(char* buf, size_t len) {
  if (!buf || len == 0) return FFB_EINVAL;
  strncpy(buf, ffb::g_last_error, len - 1);
  buf[len - 1] = 0;
  return FFB_OK;
}

int ffb_device_error(uint32_t* word, int clear) {
  if (!word) return ffb::fail(FFB_EINVAL, "ffb_device_error: word is NULL");
  cudaError_t e = cudaMemcpyFromSymbol(word, ffb_device_error_word, sizeof(uint32_t));
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_device_error: %s", cudaGetErrorString(e));
  if (clear) {
    uint32_t zero = 0;
    e = cudaMemcpyToSymbol(ffb_device_error_word, &zero, sizeof(uint32_t));
    if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_device_error: %s", cudaGetErrorString(e));
  }
  return FFB_OK;
}

}  // extern "C"
