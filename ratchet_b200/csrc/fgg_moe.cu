// fgg_moe.cu - the kernels around the expert-parallel grouped GEMM: the
// dispatch plan (a stable counting sort of the routes by destination), the
// dispatch gather (token rows -> route order) and the combine (route rows ->
// router-weighted sum per token).  Gather and combine are HBM-bound copies;
// they move 16-byte vectors with coalesced row segments and touch every
// byte once.
//
// The reference's single-GPU analogue gathers rows in `moe_gather_plan` and
// weights/sums them in `moe_combine`
// (tasks/muse_prefill_boundary/reference/submission.py:843-895).
#include <cuda_bf16.h>

#include "fgg_host.cuh"

namespace fgg {
namespace {

// One block per destination row: block r copies source row src_row[r] of
// both tensors, each thread sizeof(V) bytes at a time.
template <typename V>
__global__ void __launch_bounds__(256) gather_rows_kernel(const uint8_t* __restrict__ codes,
                                                          const uint8_t* __restrict__ sf,
                                                          const int32_t* __restrict__ src_row,
                                                          int64_t rows_in, int64_t S,
                                                          int32_t code_bytes, int32_t sf_bytes,
                                                          uint8_t* __restrict__ out_codes,
                                                          uint8_t* __restrict__ out_sf,
                                                          int* __restrict__ bad) {
  const int64_t r = blockIdx.x;
  if (r >= S) return;
  const int64_t src = src_row[r];
  if (src < 0 || src >= rows_in) {  // never read outside the source
    if (threadIdx.x == 0) atomicExch(bad, 1);
    return;
  }
  const int cw = code_bytes / int(sizeof(V));
  const V* cs = reinterpret_cast<const V*>(codes + src * code_bytes);
  V* cd = reinterpret_cast<V*>(out_codes + r * code_bytes);
  for (int i = threadIdx.x; i < cw; i += blockDim.x) cd[i] = __ldg(cs + i);
  const int sw = sf_bytes / int(sizeof(V));
  const V* ss = reinterpret_cast<const V*>(sf + src * sf_bytes);
  V* sd = reinterpret_cast<V*>(out_sf + r * sf_bytes);
  for (int i = threadIdx.x; i < sw; i += blockDim.x) sd[i] = __ldg(ss + i);
}

// out[t, :] = bf16( sum_k w[t, k] * rows[route_row[t*topk + k], :] ), fp32
// accumulation; each thread owns 8 consecutive columns (one 16-byte vector).
__global__ void __launch_bounds__(256) combine_kernel(const __nv_bfloat16* __restrict__ rows,
                                                      int64_t num_rows,
                                                      const int32_t* __restrict__ route_row,
                                                      const float* __restrict__ w, int32_t T,
                                                      int32_t topk, int32_t n,
                                                      __nv_bfloat16* __restrict__ out,
                                                      int* __restrict__ bad) {
  const int t = blockIdx.x;
  const int col = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (t >= T || col >= n) return;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  for (int k = 0; k < topk; ++k) {
    const int64_t r = route_row[int64_t(t) * topk + k];
    if (r < 0 || r >= num_rows) {
      atomicExch(bad, 1);
      continue;
    }
    const float wk = w[int64_t(t) * topk + k];
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(rows + r * n + col));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      acc[2 * j] = fmaf(wk, f.x, acc[2 * j]);
      acc[2 * j + 1] = fmaf(wk, f.y, acc[2 * j + 1]);
    }
  }
  uint4 o;
  __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
  *reinterpret_cast<uint4*>(out + int64_t(t) * n + col) = o;
}

// Dispatch plan: a stable counting sort of the routes by destination bin
// (owner rank x slot of the expert on it).  One CTA of kPlanWarps warps; warp
// w owns the contiguous route chunk [w*chunk, (w+1)*chunk) and walks it 32
// routes at a time, so the order inside a bin is the route order, as a stable
// sort would leave it.  Lanes holding the same bin in one step are grouped
// with __match_any_sync: their count goes to the warp's histogram (phase A),
// and their rank among themselves gives each one its slot (phase C).
// The expert -> bin table sits in shared memory and each walk loads kPlanUnroll
// steps of expert ids at once, so the walks are not a chain of dependent
// global loads.
constexpr int kPlanWarps = 16;
constexpr int kPlanMaxBins = 512;
constexpr int kPlanMaxExperts = 8192;
constexpr int kPlanUnroll = 8;

__global__ void __launch_bounds__(kPlanWarps * 32) plan_kernel(
    const int32_t* __restrict__ ids, int32_t routes, int32_t topk,
    const int32_t* __restrict__ owner, const int32_t* __restrict__ slot, int32_t num_experts,
    int32_t local, int32_t bins, int32_t* __restrict__ counts, int32_t* __restrict__ src_row,
    int32_t* __restrict__ route_pos, int* __restrict__ bad) {
  // [kPlanWarps][bins] warp histograms, [bins] totals, [num_experts] bin of each expert
  extern __shared__ int32_t hist[];
  int32_t* total = hist + kPlanWarps * bins;
  int32_t* ebin = total + bins;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kPlanWarps * bins; i += blockDim.x) hist[i] = 0;
  for (int e = threadIdx.x; e < num_experts; e += blockDim.x) {
    const int sl = slot[e];
    const int b = owner[e] * local + sl;
    ebin[e] = (sl < 0 || sl >= local || b < 0 || b >= bins) ? -1 : b;  // -1: bad placement
  }
  __syncthreads();
  const int chunk = (routes + kPlanWarps - 1) / kPlanWarps;
  const int lo = min(routes, warp * chunk), hi = min(routes, lo + chunk);
  // bin of route i given its expert id: -1 out of range (flagged), -2 past the chunk
  auto bin_of = [&](int i, int e) -> int {
    if (i >= hi) return -2;
    if (e < 0 || e >= num_experts) return -1;
    return ebin[e];
  };
  // A: per-warp histogram
  for (int base = lo; base < hi; base += 32 * kPlanUnroll) {
    int e[kPlanUnroll];
#pragma unroll
    for (int u = 0; u < kPlanUnroll; ++u) {
      const int i = base + 32 * u + lane;
      e[u] = i < hi ? ids[i] : 0;
    }
#pragma unroll
    for (int u = 0; u < kPlanUnroll; ++u) {
      const int b = bin_of(base + 32 * u + lane, e[u]);
      if (b == -1) atomicExch(bad, 1);
      const unsigned same = __match_any_sync(0xffffffffu, b);
      if (b >= 0 && lane == __ffs(same) - 1) hist[warp * bins + b] += __popc(same);
      __syncwarp();
    }
  }
  __syncthreads();
  // B: bin totals, exclusive offsets over bins, per-warp bases within a bin
  for (int b = threadIdx.x; b < bins; b += blockDim.x) {
    int acc = 0;
    for (int w = 0; w < kPlanWarps; ++w) acc += hist[w * bins + b];
    total[b] = acc;
    counts[b] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // bins <= kPlanMaxBins: a serial scan is a few microseconds
    int run = 0;
    for (int b = 0; b < bins; ++b) {
      const int c = total[b];
      total[b] = run;
      run += c;
    }
  }
  __syncthreads();
  for (int b = threadIdx.x; b < bins; b += blockDim.x) {
    int run = total[b];
    for (int w = 0; w < kPlanWarps; ++w) {
      const int c = hist[w * bins + b];
      hist[w * bins + b] = run;
      run += c;
    }
  }
  __syncthreads();
  // C: positions, in the same walk order as A
  for (int base = lo; base < hi; base += 32 * kPlanUnroll) {
    int e[kPlanUnroll];
#pragma unroll
    for (int u = 0; u < kPlanUnroll; ++u) {
      const int i = base + 32 * u + lane;
      e[u] = i < hi ? ids[i] : 0;
    }
#pragma unroll
    for (int u = 0; u < kPlanUnroll; ++u) {
      const int i = base + 32 * u + lane;
      const int b = bin_of(i, e[u]);
      const unsigned same = __match_any_sync(0xffffffffu, b);
      int pos = -1;
      if (b >= 0) pos = hist[warp * bins + b] + __popc(same & ((1u << lane) - 1u));
      __syncwarp();
      if (b >= 0 && lane == __ffs(same) - 1) hist[warp * bins + b] += __popc(same);
      __syncwarp();
      if (i < hi) {
        route_pos[i] = pos;
        if (pos >= 0) src_row[pos] = i / topk;
      }
    }
  }
}

}  // namespace
}  // namespace fgg

using namespace fgg;

extern "C" {

int fgg_moe_gather_rows(const void* codes, const void* sf, int64_t rows_in, int32_t code_bytes,
                        int32_t sf_bytes, const int32_t* src_row, int64_t num_rows,
                        void* out_codes, void* out_sf, int* bad, void* stream) {
  if (num_rows < 0 || rows_in < 0 || code_bytes <= 0 || sf_bytes <= 0)
    return set_error(FGG_EINVAL, "negative row count or non-positive row size");
  if (num_rows == 0) return FGG_OK;
  if (codes == nullptr || sf == nullptr || src_row == nullptr || out_codes == nullptr ||
      out_sf == nullptr || bad == nullptr)
    return set_error(FGG_EINVAL, "null pointer");
  if (num_rows > INT32_MAX) return set_error(FGG_EBADSHAPE, "too many rows");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool vec16 = code_bytes % 16 == 0 && sf_bytes % 16 == 0 && aligned16(codes) &&
                     aligned16(sf) && aligned16(out_codes) && aligned16(out_sf);
  const bool vec4 = code_bytes % 4 == 0 && sf_bytes % 4 == 0 && aligned4(codes) &&
                    aligned4(sf) && aligned4(out_codes) && aligned4(out_sf);
  const auto* c = static_cast<const uint8_t*>(codes);
  const auto* f = static_cast<const uint8_t*>(sf);
  auto* oc = static_cast<uint8_t*>(out_codes);
  auto* of = static_cast<uint8_t*>(out_sf);
  if (vec16)
    gather_rows_kernel<uint4><<<unsigned(num_rows), 256, 0, s>>>(c, f, src_row, rows_in, num_rows,
                                                                 code_bytes, sf_bytes, oc, of, bad);
  else if (vec4)
    gather_rows_kernel<uint32_t><<<unsigned(num_rows), 256, 0, s>>>(
        c, f, src_row, rows_in, num_rows, code_bytes, sf_bytes, oc, of, bad);
  else
    return set_error(FGG_EALIGN, "row sizes and pointers must be multiples of 4 bytes");
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

int fgg_moe_plan(const int32_t* topk_ids, int32_t num_tokens, int32_t topk,
                 const int32_t* owner, const int32_t* slot, int32_t num_experts, int32_t world,
                 int32_t local, int32_t* counts, int32_t* src_row, int32_t* route_pos, int* bad,
                 void* stream) {
  if (num_tokens < 0 || topk < 1 || num_experts < 1 || world < 1 || local < 1)
    return set_error(FGG_EINVAL, "bad plan sizes");
  const int64_t bins = int64_t(world) * local;
  if (bins > kPlanMaxBins)
    return set_error(FGG_EBADSHAPE, "world x local experts = %lld exceeds %d", (long long)bins,
                     kPlanMaxBins);
  if (num_experts > kPlanMaxExperts)
    return set_error(FGG_EBADSHAPE, "num_experts = %d exceeds %d", num_experts, kPlanMaxExperts);
  const int64_t routes = int64_t(num_tokens) * topk;
  if (routes > INT32_MAX) return set_error(FGG_EBADSHAPE, "too many routes");
  if (topk_ids == nullptr || owner == nullptr || slot == nullptr || counts == nullptr ||
      src_row == nullptr || route_pos == nullptr || bad == nullptr)
    return set_error(FGG_EINVAL, "null pointer");
  const size_t smem =
      (size_t(kPlanWarps + 1) * size_t(bins) + size_t(num_experts)) * sizeof(int32_t);
  if (smem > 48 * 1024)
    FGG_CUDA_CHECK(cudaFuncSetAttribute(plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        int(smem)));
  plan_kernel<<<1, kPlanWarps * 32, smem, reinterpret_cast<cudaStream_t>(stream)>>>(
      topk_ids, int32_t(routes), topk, owner, slot, num_experts, local, int32_t(bins), counts,
      src_row, route_pos, bad);
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

int fgg_moe_combine(const void* rows, int64_t num_rows, const int32_t* route_row,
                    const float* weights, int32_t num_tokens, int32_t topk, int32_t n, void* out,
                    int* bad, void* stream) {
  if (num_tokens < 0 || topk < 1 || n <= 0 || n % 8 != 0)
    return set_error(FGG_EBADSHAPE, "need num_tokens >= 0, topk >= 1, n a positive multiple of 8");
  if (num_tokens == 0) return FGG_OK;
  if (rows == nullptr || route_row == nullptr || weights == nullptr || out == nullptr ||
      bad == nullptr)
    return set_error(FGG_EINVAL, "null pointer");
  if (!aligned16(rows) || !aligned16(out))
    return set_error(FGG_EALIGN, "rows and out must be 16-byte aligned");
  const dim3 grid(unsigned(num_tokens), unsigned((n / 8 + 255) / 256));
  combine_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(rows), num_rows, route_row, weights, num_tokens, topk, n,
      static_cast<__nv_bfloat16*>(out), bad);
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

}  // extern "C"
