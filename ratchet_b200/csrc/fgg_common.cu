// fgg_common.cu - error reporting, device checks, tensor-map encoding and the
// status read-back shared by all entry points.
#include "fgg_host.cuh"

#include <atomic>
#include <cstring>
#include <mutex>

namespace fgg {

namespace {
thread_local char g_detail[512] = "";

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
int g_encode_status = FGG_OK;

void load_encoder() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) {
    g_encode_status = FGG_ECUDA;
    return;
  }
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}

DeviceInfo g_devs[64];
std::mutex g_dev_mu;

// Driver entry points for the current context and its unique id (fetched
// through the runtime, like the tensor-map encoder).
using PfnCtxGetCurrent = CUresult (*)(CUcontext*);
using PfnCtxGetId = CUresult (*)(CUcontext, unsigned long long*);
PfnCtxGetCurrent g_ctx_current = nullptr;
PfnCtxGetId g_ctx_id = nullptr;
std::once_flag g_ctx_once;

void load_ctx_entry_points() {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
  if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_ctx_current = reinterpret_cast<PfnCtxGetCurrent>(fn);
  fn = nullptr;
  if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_ctx_id = reinterpret_cast<PfnCtxGetId>(fn);
}

// Kernels whose dynamic shared-memory limit was raised, per context.
struct AttrEntry {
  const void* func = nullptr;
  uint64_t ctx = 0;
};
constexpr int kAttrSlots = 64;
AttrEntry g_attr[kAttrSlots];
int g_attr_next = 0;
std::mutex g_attr_mu;
}  // namespace

namespace {
std::atomic<int32_t> g_debug_flags{0};
}  // namespace

int32_t debug_flags() { return g_debug_flags.load(std::memory_order_relaxed); }

uint64_t current_context_id() {
  std::call_once(g_ctx_once, load_ctx_entry_points);
  if (g_ctx_current == nullptr || g_ctx_id == nullptr) return 0;
  CUcontext c = nullptr;
  if (g_ctx_current(&c) != CUDA_SUCCESS || c == nullptr) return 0;
  unsigned long long id = 0;
  if (g_ctx_id(c, &id) != CUDA_SUCCESS) return 0;
  return uint64_t(id) + 1;  // never 0 for a live context
}

int ensure_max_dynamic_smem(const void* func, int bytes) {
  const uint64_t ctx = current_context_id();
  std::lock_guard<std::mutex> lk(g_attr_mu);
  if (ctx != 0)
    for (const AttrEntry& e : g_attr)
      if (e.func == func && e.ctx == ctx) return FGG_OK;
  FGG_CUDA_CHECK(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  // the call above initialises the context if nothing had yet
  const uint64_t now = ctx != 0 ? ctx : current_context_id();
  if (now != 0) {
    g_attr[g_attr_next] = AttrEntry{func, now};
    g_attr_next = (g_attr_next + 1) % kAttrSlots;
  }
  return FGG_OK;
}

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_detail, sizeof(g_detail), fmt, ap);
  va_end(ap);
  return code;
}

int current_device(DeviceInfo* out) {
  int dev = -1;
  FGG_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return set_error(FGG_EINVAL, "device ordinal %d out of range", dev);
  {
    std::lock_guard<std::mutex> lk(g_dev_mu);
    DeviceInfo& d = g_devs[dev];
    if (d.device != dev) {
      FGG_CUDA_CHECK(cudaDeviceGetAttribute(&d.sm_count, cudaDevAttrMultiProcessorCount, dev));
      FGG_CUDA_CHECK(cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev));
      FGG_CUDA_CHECK(cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev));
      FGG_CUDA_CHECK(
          cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
      d.device = dev;
    }
    *out = d;
  }
  if (out->major != 10 || out->minor != 0)
    return set_error(FGG_EARCH, "device %d is sm_%d%d; this library is built for sm_100a", dev,
                     out->major, out->minor);
  return FGG_OK;
}

// The encoder's arguments, which fully determine its result: a repeated call
// (the same buffers every step) copies the remembered map instead of
// encoding again.  Per host thread, a few entries replaced round-robin.
struct EncodeKey {
  int dtype, rank, swz;
  const void* base;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  bool operator==(const EncodeKey& o) const { return memcmp(this, &o, sizeof(*this)) == 0; }
};
struct EncodeMemo {
  static constexpr int kEntries = 64;
  EncodeKey key[kEntries];
  CUtensorMap map[kEntries];
  bool used[kEntries];
  int next;
};
static thread_local EncodeMemo t_memo;

static int encode(CUtensorMap* out, CUtensorMapDataType dtype, cuuint32_t rank, const void* base,
                  const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                  CUtensorMapSwizzle swz) {
  EncodeKey k;
  memset(&k, 0, sizeof(k));  // padding too: keys compare as bytes
  k.dtype = int(dtype);
  k.rank = int(rank);
  k.swz = int(swz);
  k.base = base;
  for (cuuint32_t i = 0; i < rank && i < 3; ++i) {
    k.dims[i] = dims[i];
    k.box[i] = box[i];
    if (i + 1 < rank) k.strides[i] = strides[i];
  }
  EncodeMemo& m = t_memo;
  if (rank <= 3) {
    for (int i = 0; i < EncodeMemo::kEntries; ++i)
      if (m.used[i] && m.key[i] == k) {
        *out = m.map[i];
        return FGG_OK;
      }
  }
  std::call_once(g_encode_once, load_encoder);
  if (g_encode == nullptr)
    return set_error(FGG_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = g_encode(out, dtype, rank, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(FGG_ECUDA, "cuTensorMapEncodeTiled failed (CUresult %d, rank %u)", int(r),
                     rank);
  if (rank <= 3) {
    const int i = m.next;
    m.next = (m.next + 1) % EncodeMemo::kEntries;
    m.key[i] = k;
    m.map[i] = *out;
    m.used[i] = true;
  }
  return FGG_OK;
}

int encode_u8_2d(CUtensorMap* out, const void* base, uint64_t inner_bytes, uint64_t rows,
                 uint32_t box_inner, uint32_t box_rows) {
  cuuint64_t dims[2] = {inner_bytes, rows};
  cuuint64_t strides[1] = {inner_bytes};
  cuuint32_t box[2] = {box_inner, box_rows};
  return encode(out, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box,
                CU_TENSOR_MAP_SWIZZLE_128B);
}

int encode_2d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base, uint64_t d0,
              uint64_t d1, uint64_t stride1_bytes, uint32_t b0, uint32_t b1) {
  cuuint64_t dims[2] = {d0, d1};
  cuuint64_t strides[1] = {stride1_bytes};
  cuuint32_t box[2] = {b0, b1};
  return encode(out, dtype, 2, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

int encode_u64_rows(CUtensorMap* out, const void* base, uint64_t rows, uint32_t row_u64,
                    uint32_t box_rows) {
  cuuint64_t dims[2] = {row_u64, rows};
  cuuint64_t strides[1] = {uint64_t(row_u64) * 8u};
  cuuint32_t box[2] = {row_u64, box_rows};
  return encode(out, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, base, dims, strides, box,
                CU_TENSOR_MAP_SWIZZLE_NONE);
}

int encode_3d(CUtensorMap* out, CUtensorMapDataType dtype, const void* base, uint64_t d0,
              uint64_t d1, uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes,
              uint32_t b0, uint32_t b1, uint32_t b2) {
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {b0, b1, b2};
  return encode(out, dtype, 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace fgg

extern "C" {

const char* fgg_error_string(int code) {
  switch (code) {
    case FGG_OK: return "ok";
    case FGG_EINVAL: return "invalid argument";
    case FGG_EBADSHAPE: return "unsupported shape";
    case FGG_EALIGN: return "misaligned pointer";
    case FGG_EWORKSPACE: return "workspace too small";
    case FGG_ECUDA: return "CUDA error";
    case FGG_ETIMEOUT: return "device wait timed out";
    case FGG_EARCH: return "unsupported GPU architecture";
    default: return "unknown error";
  }
}

const char* fgg_last_error_detail(void) { return fgg::g_detail; }

const char* fgg_version(void) { return "fgg 0.2.0 sm_100a"; }

int32_t fgg_debug_set_flags(int32_t flags) {
  return fgg::g_debug_flags.exchange(flags, std::memory_order_relaxed);
}

int fgg_read_device_status(const void* workspace, void* stream) {
  if (workspace == nullptr) return fgg::set_error(FGG_EINVAL, "workspace is null");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int host[4] = {0, 0, 0, 0};
  FGG_CUDA_CHECK(cudaMemcpyAsync(host, workspace, sizeof(host), cudaMemcpyDeviceToHost, s));
  FGG_CUDA_CHECK(cudaStreamSynchronize(s));
  if (host[0] != 0)
    return fgg::set_error(FGG_ETIMEOUT, "device status word 0x%x (a bounded wait gave up)",
                          host[0]);
  return FGG_OK;
}

}  // extern "C"
