// Peer memory for the tensor-parallel kernels: device allocations shared between the
// ranks' processes through CUDA IPC handles (one process per GPU), so that a kernel can
// read another rank's partial sums over NVLink.  No reference counterpart (the reference
// runs on one GPU, api.py:56-57); these replace NCCL's transport for the two reductions of
// each tensor-parallel decoder layer.
#include "common.cuh"

#include <string.h>

extern "C" int ffb_peer_alloc(size_t bytes, void** dptr, void* handle) {
  FFB_REQUIRE(dptr && handle && bytes > 0, "ffb_peer_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_peer_alloc: cudaMalloc: %s", cudaGetErrorString(e));
  e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return ffb::fail(FFB_ECUDA, "ffb_peer_alloc: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  *dptr = p;
  return FFB_OK;
}

extern "C" int ffb_peer_open(const void* handle, void** dptr) {
  FFB_REQUIRE(dptr && handle, "ffb_peer_open: NULL argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(dptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_peer_open: %s", cudaGetErrorString(e));
  return FFB_OK;
}

extern "C" int ffb_peer_close(void* dptr) {
  cudaError_t e = cudaIpcCloseMemHandle(dptr);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_peer_close: %s", cudaGetErrorString(e));
  return FFB_OK;
}

extern "C" int ffb_peer_free(void* dptr) {
  cudaError_t e = cudaFree(dptr);
  if (e != cudaSuccess) return ffb::fail(FFB_ECUDA, "ffb_peer_free: %s", cudaGetErrorString(e));
  return FFB_OK;
}
