// fgg_peer.cu - peer memory for the expert-parallel exchange: device buffers
// shared between the ranks of one node through CUDA IPC (an ordinary
// allocation mapped into the other processes; no multicast object), so that
// the dispatch and combine kernels store straight into their peers' buffers
// over NVLink.
#include "fgg_host.cuh"

#include <cstring>

extern "C" {

int fgg_peer_alloc(size_t bytes, void** ptr) {
  if (ptr == nullptr || bytes == 0) return fgg::set_error(FGG_EINVAL, "null pointer or zero size");
  void* p = nullptr;
  FGG_CUDA_CHECK(cudaMalloc(&p, bytes));
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return fgg::set_error(FGG_ECUDA, "cudaMemset of a peer buffer failed");
  }
  *ptr = p;
  return FGG_OK;
}

int fgg_peer_free(void* ptr) {
  if (ptr == nullptr) return FGG_OK;
  FGG_CUDA_CHECK(cudaFree(ptr));
  return FGG_OK;
}

size_t fgg_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

int fgg_peer_export(const void* ptr, void* handle) {
  if (ptr == nullptr || handle == nullptr) return fgg::set_error(FGG_EINVAL, "null pointer");
  cudaIpcMemHandle_t h;
  FGG_CUDA_CHECK(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)));
  memcpy(handle, &h, sizeof(h));
  return FGG_OK;
}

int fgg_peer_import(const void* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return fgg::set_error(FGG_EINVAL, "null pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  FGG_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = p;
  return FGG_OK;
}

int fgg_peer_close(void* ptr) {
  if (ptr == nullptr) return FGG_OK;
  FGG_CUDA_CHECK(cudaIpcCloseMemHandle(ptr));
  return FGG_OK;
}

}  // extern "C"
