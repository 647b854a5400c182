// fgg_scratch.cu - the fixed device scratch array behind
// fgg_nvfp4_grouped_gemm_noalloc.
//
// The array sits in its own translation unit, hence its own CUDA module: under
// lazy module loading a process that never calls the no-alloc entry point
// never loads it, so the other entry points pay nothing for it.
#include "fgg_host.cuh"

#include <atomic>

namespace fgg {
namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[FGG_NOALLOC_SCRATCH_BYTES];

// the array's device address per device ordinal, 0 until first looked up
std::atomic<uintptr_t> g_scratch_addr[64];

}  // namespace

int noalloc_scratch(void** out) {
  int dev = -1;
  FGG_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(FGG_EINVAL, "device ordinal %d out of range", dev);
  uintptr_t a = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (a == 0) {
    // Two threads racing here both store the same address.
    void* p = nullptr;
    FGG_CUDA_CHECK(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    a = reinterpret_cast<uintptr_t>(p);
    g_scratch_addr[dev].store(a, std::memory_order_release);
  }
  *out = reinterpret_cast<void*>(a);
  return FGG_OK;
}

}  // namespace fgg
