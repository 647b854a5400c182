// fgg_scratch.cu - the fixed device scratch array behind
// fgg_nvfp4_grouped_gemm_noalloc.
//
// The array sits in its own translation unit, hence its own CUDA module: under
// lazy module loading a process that never calls the no-alloc entry point
// never loads it, so the other entry points pay nothing for it.
#include "fgg_host.cuh"

#include <mutex>

namespace fgg {
namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[FGG_NOALLOC_SCRATCH_BYTES];

// The array's device address as looked up in one context.  A __device__
// symbol's address belongs to the context that loaded the module: after
// cudaDeviceReset, or under another context on the same device, it must be
// looked up again, so each device's entry remembers the context id it holds.
struct ScratchSlot {
  uint64_t ctx = 0;
  void* addr = nullptr;
};
ScratchSlot g_slots[64];
std::mutex g_mu;

}  // namespace

int noalloc_scratch(void** out) {
  int dev = -1;
  FGG_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(FGG_EINVAL, "device ordinal %d out of range", dev);
  const uint64_t ctx = current_context_id();
  std::lock_guard<std::mutex> lk(g_mu);
  ScratchSlot& s = g_slots[dev];
  if (ctx == 0 || s.ctx != ctx || s.addr == nullptr) {
    // set-up on this device and context: the lookup also loads the module
    void* p = nullptr;
    FGG_CUDA_CHECK(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    s.addr = p;
    s.ctx = ctx != 0 ? ctx : current_context_id();  // the lookup made a context current
  }
  *out = s.addr;
  return FGG_OK;
}

}  // namespace fgg
