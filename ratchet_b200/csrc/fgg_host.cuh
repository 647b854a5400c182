// fgg_host.cuh - host-side helpers shared by the entry points: per-thread
// error detail, the driver's tensor-map encoder (fetched through the runtime,
// so the library does not link libcuda), device capability checks and the
// workspace carving helper.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <cstdio>

#include "fgg_api.h"  // include/ is on the include path

namespace fgg {

// Set the calling thread's error detail and return `code`.
int set_error(int code, const char* fmt, ...);

#define FGG_CUDA_CHECK(expr)                                                        \
  do {                                                                              \
    cudaError_t e__ = (expr);                                                       \
    if (e__ != cudaSuccess)                                                         \
      return ::fgg::set_error(FGG_ECUDA, "%s failed: %s", #expr, cudaGetErrorString(e__)); \
  } while (0)

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
  int major = 0;
  int minor = 0;
  int max_smem_optin = 0;
};

// Current device's properties (cached per device); FGG_EARCH unless sm_100.
int current_device(DeviceInfo* out);

// Unique id of the calling thread's current CUDA context (never reused, so a
// context created after cudaDeviceReset gets a new one); 0 when no context is
// current yet.  Per-context state (a __device__ symbol's address, a kernel's
// raised shared-memory limit) is cached under this id.
uint64_t current_context_id();

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, context).
int ensure_max_dynamic_smem(const void* func, int bytes);

// Test hooks set by fgg_debug_set_flags (0 in normal use), copied into every
// GEMM launch's parameters.
int32_t debug_flags();

// 2-D uint8 tensor map, 128-byte swizzle, zero fill out of bounds:
// dims {inner_bytes, rows}, row pitch = inner_bytes, box {box_inner, box_rows}.
int encode_u8_2d(CUtensorMap* out, const void* base, uint64_t inner_bytes, uint64_t rows,
                 uint32_t box_inner, uint32_t box_rows);
// 3-D uint8 tensor map (for the MX weight tensor with a 4-bit-unpacking type).
int encode_3d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base, uint64_t d0,
              uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
              uint32_t b0, uint32_t b1, uint32_t b2);
int encode_2d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base, uint64_t d0,
              uint64_t d1, uint64_t stride1_bytes, uint32_t b0, uint32_t b1);
// A contiguous byte buffer viewed as `rows` rows of `row_u64` uint64 values,
// unswizzled, box {row_u64, box_rows}: how packed scale-factor atoms travel.
int encode_u64_rows(CUtensorMap* out, const void* base, uint64_t rows, uint32_t row_u64,
                    uint32_t box_rows);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Launch `kernel` as a programmatic dependent of the preceding kernel on the
// stream (programmatic dependent launch): it may start while that kernel
// finishes and must call griddepcontrol.wait before reading its results.
template <class... KArgs, class... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

// Sequential carve-out of one caller-owned buffer.
struct Carver {
  size_t off = 0;
  size_t take(size_t bytes, size_t align = 256) {
    off = align_up(off, align);
    const size_t at = off;
    off += bytes;
    return at;
  }
};

// Status words at the head of every workspace: [0] status code, [1] tile
// counter, [2] launch count (debug), [3] reserved.
constexpr size_t kStatusBytes = 256;

}  // namespace fgg
