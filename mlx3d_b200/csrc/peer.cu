// Device buffers shared between the processes of one node (CUDA IPC), for
// kernels that read other GPUs' memory directly over NVLink (peer loads; no
// TMA, no multicast).  The exporting process allocates with gs_peer_alloc
// and hands the 64-byte handle to the others (through the process group's
// store or an all-gather); each of them maps it with gs_peer_open.  The
// mapping is valid while the exporter keeps the buffer: close every mapping
// (gs_peer_close) before the exporter frees it (gs_peer_free).
#include <string.h>

#include "gs_common.cuh"

static_assert(sizeof(cudaIpcMemHandle_t) == GS_PEER_HANDLE_BYTES, "IPC handle size");

extern "C" {

int gs_peer_alloc(size_t bytes, void** dev_ptr, void* handle) {
  gs::clear_error();
  if (!dev_ptr || !handle) return gs::set_error(GS_ERR_INVALID_ARG, "gs_peer_alloc: NULL pointer");
  *dev_ptr = nullptr;
  if (bytes == 0) return gs::set_error(GS_ERR_INVALID_ARG, "gs_peer_alloc: zero bytes");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return gs::set_error(GS_ERR_CUDA, "gs_peer_alloc: cudaMalloc: %s", cudaGetErrorString(e));
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return gs::set_error(GS_ERR_CUDA, "gs_peer_alloc: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  *dev_ptr = p;
  return GS_OK;
}

int gs_peer_open(const void* handle, void** dev_ptr) {
  gs::clear_error();
  if (!dev_ptr || !handle) return gs::set_error(GS_ERR_INVALID_ARG, "gs_peer_open: NULL pointer");
  *dev_ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return gs::set_error(GS_ERR_CUDA, "gs_peer_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *dev_ptr = p;
  return GS_OK;
}

int gs_peer_close(void* dev_ptr) {
  gs::clear_error();
  if (!dev_ptr) return GS_OK;
  cudaError_t e = cudaIpcCloseMemHandle(dev_ptr);
  if (e != cudaSuccess) return gs::set_error(GS_ERR_CUDA, "gs_peer_close: %s", cudaGetErrorString(e));
  return GS_OK;
}

int gs_peer_free(void* dev_ptr) {
  gs::clear_error();
  if (!dev_ptr) return GS_OK;
  cudaError_t e = cudaFree(dev_ptr);
  if (e != cudaSuccess) return gs::set_error(GS_ERR_CUDA, "gs_peer_free: %s", cudaGetErrorString(e));
  return GS_OK;
}

}  // extern "C"
