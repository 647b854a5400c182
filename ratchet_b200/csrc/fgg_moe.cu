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

#include <algorithm>
#include <type_traits>
#include <cstring>

#include "fgg_host.cuh"
#include "fgg_ptx.cuh"

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

// ---- the expert-parallel layer without a host synchronisation -------------
//
// The dispatch may send any token of a rank to any rank, so an exchange
// buffer that can never overflow gives each (source, destination) pair room
// for all of the source's tokens.  At that capacity the dispatch moves the
// bytes of an all-gather of the tokens: every token leaves its rank once as
// one record (codes, scales, expert ids, router weights, decode scale) and
// each rank expands the routes of its own experts.  The combine sends one
// router-weighted partial row per (token, rank) back along an equal-split
// all-to-all and the token's rank sums those rows in fp32.  No size ever has
// to reach the host, so nothing in the layer synchronises it.

struct MoeTok {
  const uint8_t* codes;
  const uint8_t* sf;
  const uint8_t* ids;
  const uint8_t* weights;
  const uint8_t* scale;
  int64_t codes_stride, sf_stride, ids_stride, weights_stride, scale_stride;
  int32_t num_tokens, topk, k;
  const int64_t* epoch;  // double-buffered view: pointers advance by the epoch parity
  int64_t parity_bytes;
};

// The view of this forward's buffer half (a plain view is returned as it is).
__device__ __forceinline__ MoeTok resolved(MoeTok t) {
  if (t.epoch != nullptr) {
    const int64_t off = ((*t.epoch + 1) & 1) * t.parity_bytes;
    t.codes += off;
    t.sf += off;
    t.ids += off;
    if (t.weights != nullptr) t.weights += off;
    if (t.scale != nullptr) t.scale += off;
    t.epoch = nullptr;
  }
  return t;
}

__device__ __forceinline__ int32_t tok_id(const MoeTok& t, int64_t i, int k) {
  return __ldg(reinterpret_cast<const int32_t*>(t.ids + i * t.ids_stride) + k);
}
__device__ __forceinline__ float tok_weight(const MoeTok& t, int64_t i, int k) {
  return t.weights == nullptr
             ? 1.0f
             : __ldg(reinterpret_cast<const float*>(t.weights + i * t.weights_stride) + k);
}
__device__ __forceinline__ float tok_scale(const MoeTok& t, int64_t i) {
  return t.scale == nullptr ? 1.0f
                            : __ldg(reinterpret_cast<const float*>(t.scale + i * t.scale_stride));
}

// Copy `bytes` (a multiple of 16, both ends 16-byte aligned) with the calling
// warp: each lane moves every 32nd 16-byte vector.
__device__ __forceinline__ void warp_copy16(uint8_t* __restrict__ dst,
                                            const uint8_t* __restrict__ src, int bytes) {
  const int n = bytes / 16;
  for (int i = threadIdx.x & 31; i < n; i += 32)
    reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
}
// Same with 4-byte words (multiples of 4, 4-byte aligned).
__device__ __forceinline__ void warp_copy4(uint8_t* __restrict__ dst,
                                           const uint8_t* __restrict__ src, int bytes) {
  const int n = bytes / 4;
  for (int i = threadIdx.x & 31; i < n; i += 32)
    reinterpret_cast<uint32_t*>(dst)[i] = __ldg(reinterpret_cast<const uint32_t*>(src) + i);
}

// One token record per warp: [codes K/2][scales K/16][ids topk][weights topk][scale].
template <bool kVec>
__global__ void __launch_bounds__(256) moe_pack_kernel(MoeTok t, uint8_t* __restrict__ rec,
                                                       int64_t rec_bytes) {
  const int64_t i = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  if (i >= t.num_tokens) return;
  const int lane = threadIdx.x & 31;
  uint8_t* r = rec + i * rec_bytes;
  const int kh = t.k / 2, ks = t.k / 16;
  if (kVec) {
    warp_copy16(r, t.codes + i * t.codes_stride, kh);
    warp_copy16(r + kh, t.sf + i * t.sf_stride, ks);
  } else {
    warp_copy4(r, t.codes + i * t.codes_stride, kh);
    warp_copy4(r + kh, t.sf + i * t.sf_stride, ks);
  }
  int32_t* ids = reinterpret_cast<int32_t*>(r + kh + ks);
  float* w = reinterpret_cast<float*>(ids + t.topk);
  for (int k = lane; k < t.topk; k += 32) {
    ids[k] = tok_id(t, i, k);
    w[k] = tok_weight(t, i, k);
  }
  if (lane == 0) w[t.topk] = tok_scale(t, i);
}

// Expand: the routes of this rank's experts, placed expert by expert into
// one buffer of token rows.  Two kernels over the routes, many blocks each:
//   count  per-block histograms of the local routes by slot, added into
//          counts[slot] (zeroed before the launch)
//   place  every block scans counts into offsets (block 0 publishes them for
//          the GEMM); then one warp per route: a local route takes the next
//          row of its expert (atomic cursor), records it in route_row, and the
//          warp copies the token's codes and scales into that row.
// Route (i, k) to another rank's expert, or absent (expert id < 0, e.g. a
// padding token's), gets route_row -1; an expert id >= E or a placement
// outside the local slots sets *bad = 1 and gets -1.  The row order inside an
// expert follows the atomics: each expanded row is computed on its own and
// summed back in route order, so the results do not depend on it.
constexpr int kExpandMaxLocal = 1024;

__device__ __forceinline__ int local_slot_of(const MoeTok& t, int64_t r,
                                             const int32_t* __restrict__ owner,
                                             const int32_t* __restrict__ slot, int num_experts,
                                             int rank, int local, int* bad) {
  const int e = tok_id(t, r / t.topk, int(r % t.topk));
  if (e < 0) return -1;  // an absent route
  if (e >= num_experts) {
    atomicExch(bad, 1);
    return -1;
  }
  if (__ldg(owner + e) != rank) return -1;
  const int s = __ldg(slot + e);
  if (s < 0 || s >= local) {
    atomicExch(bad, 1);
    return -1;
  }
  return s;
}

__global__ void __launch_bounds__(256)
    moe_expand_count_kernel(MoeTok t, const int32_t* __restrict__ owner,
                            const int32_t* __restrict__ slot, int32_t num_experts, int32_t rank,
                            int32_t local, int32_t* __restrict__ counts, int* __restrict__ bad) {
  griddep_wait();
  t = resolved(t);
  __shared__ int32_t hist[kExpandMaxLocal];
  for (int i = threadIdx.x; i < local; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const int64_t routes = int64_t(t.num_tokens) * t.topk;
  for (int64_t r = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; r < routes;
       r += int64_t(gridDim.x) * blockDim.x) {
    const int s = local_slot_of(t, r, owner, slot, num_experts, rank, local, bad);
    if (s >= 0) atomicAdd(&hist[s], 1);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < local; i += blockDim.x)
    if (hist[i]) atomicAdd(counts + i, hist[i]);
  griddep_launch_dependents();
}

template <bool kVec>
__global__ void __launch_bounds__(256)
    moe_expand_place_kernel(MoeTok t, const int32_t* __restrict__ owner,
                            const int32_t* __restrict__ slot, int32_t num_experts, int32_t rank,
                            int32_t local, int32_t max_rows, const int32_t* __restrict__ counts,
                            int32_t* __restrict__ cursor, int32_t* __restrict__ offsets,
                            int32_t* __restrict__ route_row, int32_t* __restrict__ src_token,
                            float* __restrict__ row_scale, uint8_t* __restrict__ out_codes,
                            uint8_t* __restrict__ out_sf, int* __restrict__ bad) {
  griddep_wait();
  t = resolved(t);
  __shared__ int32_t base[kExpandMaxLocal + 1];
  if (threadIdx.x == 0) {  // local <= 1024: a serial scan of the counts
    int run = 0;
    for (int s = 0; s < local; ++s) {
      base[s] = run;
      run += counts[s];
    }
    base[local] = run;
  }
  __syncthreads();
  if (blockIdx.x == 0)
    for (int s = threadIdx.x; s <= local; s += blockDim.x) offsets[s] = min(base[s], max_rows);
  const int lane = threadIdx.x & 31;
  const int kh = t.k / 2, ks = t.k / 16;
  const int64_t routes = int64_t(t.num_tokens) * t.topk;
  const int64_t warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  for (int64_t r = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < routes; r += warps) {
    int row = -1;
    if (lane == 0) {
      const int s = local_slot_of(t, r, owner, slot, num_experts, rank, local, bad);
      if (s >= 0) {
        row = base[s] + atomicAdd(cursor + s, 1);
        if (row >= max_rows) {  // the caller's buffer is too small: flag, drop
          atomicExch(bad, 2);
          row = -1;
        }
      }
      route_row[r] = row;
    }
    row = __shfl_sync(0xffffffffu, row, 0);
    if (row < 0) continue;
    const int64_t tok = r / t.topk;
    if (lane == 0) {
      src_token[row] = int32_t(tok);
      row_scale[row] = tok_scale(t, tok);
    }
    if (kVec) {
      warp_copy16(out_codes + int64_t(row) * kh, t.codes + tok * t.codes_stride, kh);
      warp_copy16(out_sf + int64_t(row) * ks, t.sf + tok * t.sf_stride, ks);
    } else {
      warp_copy4(out_codes + int64_t(row) * kh, t.codes + tok * t.codes_stride, kh);
      warp_copy4(out_sf + int64_t(row) * ks, t.sf + tok * t.sf_stride, ks);
    }
  }
  griddep_launch_dependents();
}

// ---- peer exchange (see fgg_api.h): buffers mapped from the other ranks ----
constexpr int kPeersMax = FGG_PEERS_MAX;
constexpr int kStatusPeerTimeout = 0x301;
// A peer's flag waits on the other ranks' hosts too (their launches of the
// same forward), so its default limit is longer than a kernel-internal wait's.
constexpr int32_t kPeerWaitDefaultMs = 10000;

struct PeerDev {
  int32_t world, rank, capacity, n;
  int64_t* epoch;
  int32_t* counters;  // [0] dispatch, [1] combine, [2] sum: blocks done
  int* status;
  uint8_t* gathered[kPeersMax];
  uint8_t* recv[kPeersMax];
  unsigned long long* flags[kPeersMax];  // [2][kPeersMax] per rank
  const int32_t* owner;                  // [num_experts] rank of each expert
  int32_t num_experts;
  int32_t* routes;                       // [capacity] destination ranks per token slot
  uint64_t wait_ns;                      // limit of each wait on the peers' flags
  int64_t rb;                            // record bytes
  int64_t gathered_half;                 // bytes of one buffer half
};

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Called by every thread of every block once its stores are issued: the last
// block to finish raises this forward's flag of `kind` in every rank.  The
// barrier orders the block's stores before thread 0's system-scope fence,
// whose cumulativity covers them, so one fence per block releases them all
// (the pattern of a grid-wide barrier, here at system scope).
__device__ __forceinline__ void signal_peers(const PeerDev& x, int kind, unsigned long long e) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();  // the block's stores, to every rank, before the count
    const unsigned nblocks = gridDim.x * gridDim.y;
    const int prev = atomicAdd(x.counters + kind, 1);
    if (unsigned(prev) == nblocks - 1) {
      x.counters[kind] = 0;  // the next forward's count starts from zero (stream order)
      __threadfence_system();
      for (int s = 0; s < x.world; ++s) st_release_sys(x.flags[s] + kind * kPeersMax + x.rank, e);
    }
  }
}

// Router-weighted sum of one token's local routes over 8 columns:
// bf16(sum_k w[i, k] * rows[route_row[i * topk + k], col:col+8]) over the
// routes with a row (>= 0), fp32 accumulation in route order; *any tells
// whether the token has a route here at all.
__device__ __forceinline__ uint4 reduce_routes(const MoeTok& t, const __nv_bfloat16* rows,
                                               int32_t num_rows, const int32_t* route_row,
                                               int32_t n, int64_t i, int col, int* bad,
                                               bool* any) {
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  bool seen = false;
  for (int k = 0; k < t.topk; ++k) {
    const int r = __ldg(route_row + i * t.topk + k);
    if (r < 0) continue;
    if (r >= num_rows) {
      atomicExch(bad, 1);
      continue;
    }
    seen = true;
    const float wk = tok_weight(t, i, k);
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(rows + int64_t(r) * n + col));
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
  *any = seen;
  return o;
}

// out[i, :] = the router-weighted sum of token i's local routes: block (i, y)
// takes 8 columns a thread, so that many blocks stay resident to hide the row
// loads' latency.  A token with no local route gets a zero row, or no row at
// all with skip_empty (its reader knows, from the routes, not to read it).
__global__ void __launch_bounds__(256) moe_reduce_kernel(MoeTok t,
                                                         const __nv_bfloat16* __restrict__ rows,
                                                         int32_t num_rows,
                                                         const int32_t* __restrict__ route_row,
                                                         int32_t n, __nv_bfloat16* __restrict__ out,
                                                         int* __restrict__ bad, int skip_empty) {
  griddep_wait();
  t = resolved(t);
  const int64_t i = blockIdx.x;
  const int col = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (i < t.num_tokens && col < n) {
    bool any;
    const uint4 o = reduce_routes(t, rows, num_rows, route_row, n, i, col, bad, &any);
    if (any || !skip_empty) *reinterpret_cast<uint4*>(out + i * n + col) = o;
  }
}

// One thread raises this forward's flag of `kind` in every rank, after the
// kernels before it on the stream: their writes to this GPU's memory are
// complete when it starts, and the fence orders them before the flags that
// peers acquire (a peer reads this GPU's memory through this GPU's L2).
__global__ void moe_signal_peers_kernel(PeerDev x, int kind) {
  if (threadIdx.x != 0) return;
  const unsigned long long e = (unsigned long long)(*x.epoch + 1);
  __threadfence_system();
  for (int s = 0; s < x.world; ++s) st_release_sys(x.flags[s] + kind * kPeersMax + x.rank, e);
}

// Dispatch over peer memory: one warp per (token slot of this rank,
// destination rank), so the stores to different ranks proceed in parallel
// and even a few hundred slots keep every SM storing.  Each warp finds the
// ranks that own one of the token's experts (a bit mask; the warp of this
// rank keeps it in routes[j]).  If its destination is among them it writes
// the whole record there (codes, scales, expert ids, router weights, decode
// scale), otherwise only expert ids -1, as for slots past the rank's tokens.
// The codes and scales are contiguous in a record, so 16-byte piece q of the
// record comes from the codes (q < K/32) or the scales; a lane loads up to
// kDispatchBatch pieces before it stores any.  The dispatch flags follow.
constexpr int kDispatchBatch = 8;

template <bool kVec>
__global__ void __launch_bounds__(256) moe_dispatch_peers_kernel(MoeTok t, PeerDev x) {
  using V = typename std::conditional<kVec, uint4, uint32_t>::type;
  constexpr int kB = int(sizeof(V));
  const unsigned long long e = (unsigned long long)(*x.epoch + 1);
  const int64_t par = int64_t(e & 1ull);
  const int lane = threadIdx.x & 31;
  const int kh = t.k / 2, ks = t.k / 16;
  const int nc = kh / kB, np = (kh + ks) / kB;  // pieces: codes, then all
  const int64_t warps = (int64_t(gridDim.x) * blockDim.x) >> 5;
  const int64_t items = int64_t(x.capacity) * x.world;
  for (int64_t w = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < items;
       w += warps) {  // warp-uniform
    const int64_t j = w / x.world;
    const int dst = int(w - j * x.world);
    uint8_t* const rec = x.gathered[dst] + par * x.gathered_half +
                         (int64_t(x.rank) * x.capacity + j) * x.rb;
    int32_t* const ids = reinterpret_cast<int32_t*>(rec + kh + ks);
    unsigned bit = 0;
    if (j < t.num_tokens) {
      for (int k = lane; k < t.topk; k += 32) {
        const int32_t id = tok_id(t, j, k);
        if (id >= 0 && id < x.num_experts) {
          const int o = __ldg(x.owner + id);
          if (o >= 0 && o < x.world) bit |= 1u << o;
        }
      }
    }
    const unsigned mask = __reduce_or_sync(0xffffffffu, bit);
    if (dst == x.rank && lane == 0) x.routes[j] = int32_t(mask);
    if (!((mask >> dst) & 1u)) {
      for (int k = lane; k < t.topk; k += 32) ids[k] = -1;
      continue;
    }
    const V* codes = reinterpret_cast<const V*>(t.codes + j * t.codes_stride);
    const V* sf = reinterpret_cast<const V*>(t.sf + j * t.sf_stride);
    V* out = reinterpret_cast<V*>(rec);
    for (int base = 0; base < np; base += 32 * kDispatchBatch) {
      V v[kDispatchBatch];
#pragma unroll
      for (int u = 0; u < kDispatchBatch; ++u) {
        const int q = base + u * 32 + lane;
        if (q < np) v[u] = q < nc ? __ldg(codes + q) : __ldg(sf + (q - nc));
      }
#pragma unroll
      for (int u = 0; u < kDispatchBatch; ++u) {
        const int q = base + u * 32 + lane;
        if (q < np) out[q] = v[u];
      }
    }
    for (int k = lane; k < t.topk; k += 32) {
      ids[k] = tok_id(t, j, k);
      reinterpret_cast<float*>(ids + t.topk)[k] = tok_weight(t, j, k);
    }
    if (lane == 0) reinterpret_cast<float*>(ids + 2 * t.topk)[0] = tok_scale(t, j);
  }
  signal_peers(x, 0, e);
}

// Bounded wait (one thread) until every rank's flag of `kind` in this rank's
// memory carries this forward's epoch; gives up after wait_ns with status
// 0x301.
__global__ void moe_wait_peers_kernel(PeerDev x, int kind) {
  if (threadIdx.x != 0) return;
  const unsigned long long e = (unsigned long long)(*x.epoch + 1);
  const unsigned long long* f = x.flags[x.rank] + kind * kPeersMax;
  const uint64_t t0 = globaltimer();
  for (int s = 0; s < x.world; ++s) {
    while (ld_acquire_sys(f + s) < e) {
      if (globaltimer() - t0 > x.wait_ns) {
        atomicCAS(x.status, 0, kStatusPeerTimeout);
        return;
      }
    }
  }
}

// out[i, :] = bf16(sum_s recv_s[rank * capacity + i, :]) over the ranks s
// in routes[i], in rank order (the others hold no row for the token): the
// partial rows are read where they were computed, over NVLink for s != rank.
// Block (i, y) takes 8 columns a thread and issues its loads from every
// source before it sums.  The last block to finish advances the epoch.
__global__ void __launch_bounds__(256) moe_sum_peers_kernel(PeerDev x, int32_t tokens,
                                                            __nv_bfloat16* __restrict__ out) {
  griddep_wait();
  const int n = x.n;
  const int64_t i = blockIdx.x;
  const int col = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (i < tokens && col < n) {
    const unsigned mask = unsigned(x.routes[i]);
    const int64_t row = int64_t(x.rank) * x.capacity + i;
    uint4 v[kPeersMax];
#pragma unroll
    for (int s = 0; s < kPeersMax; ++s)
      if (s < x.world && ((mask >> s) & 1u))
        v[s] = *reinterpret_cast<const uint4*>(
            reinterpret_cast<const __nv_bfloat16*>(x.recv[s]) + row * n + col);
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
#pragma unroll
    for (int s = 0; s < kPeersMax; ++s) {
      if (!(s < x.world && ((mask >> s) & 1u))) continue;
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v[s]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __bfloat1622float2(h[j]);
        acc[2 * j] += f.x;
        acc[2 * j + 1] += f.y;
      }
    }
    uint4 o;
    __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
    *reinterpret_cast<uint4*>(out + i * n + col) = o;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (unsigned(atomicAdd(x.counters + 2, 1)) == gridDim.x * gridDim.y - 1) {
      x.counters[2] = 0;
      *x.epoch = *x.epoch + 1;  // every block of this forward has read it
    }
  }
}

// out[i, :] = bf16(sum_s parts[s * per_source + i, :]) in fp32 (the partial
// rows every rank sent back for this rank's tokens).
__global__ void __launch_bounds__(256) moe_sum_parts_kernel(const __nv_bfloat16* __restrict__ parts,
                                                            int32_t world, int32_t per_source,
                                                            int32_t tokens, int32_t n,
                                                            __nv_bfloat16* __restrict__ out) {
  griddep_wait();
  const int64_t i = blockIdx.x;
  const int col = (blockIdx.y * blockDim.x + threadIdx.x) * 8;
  if (i >= tokens || col >= n) return;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
  for (int s = 0; s < world; ++s) {
    const uint4 v =
        __ldg(reinterpret_cast<const uint4*>(parts + (int64_t(s) * per_source + i) * n + col));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(h[j]);
      acc[2 * j] += f.x;
      acc[2 * j + 1] += f.y;
    }
  }
  uint4 o;
  __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
  *reinterpret_cast<uint4*>(out + i * n + col) = o;
}

int to_dev(const FggMoeTokens* t, MoeTok* d) {
  if (t == nullptr) return set_error(FGG_EINVAL, "tokens is null");
  if (t->num_tokens < 0 || t->topk < 1 || t->k < 64 || t->k % 64 != 0)
    return set_error(FGG_EBADSHAPE, "need num_tokens >= 0, topk >= 1, K a multiple of 64");
  if (t->num_tokens > 0 && (t->ids == nullptr))
    return set_error(FGG_EINVAL, "ids is null");
  d->codes = static_cast<const uint8_t*>(t->codes);
  d->sf = static_cast<const uint8_t*>(t->sf);
  d->ids = reinterpret_cast<const uint8_t*>(t->ids);
  d->weights = reinterpret_cast<const uint8_t*>(t->weights);
  d->scale = reinterpret_cast<const uint8_t*>(t->scale);
  d->codes_stride = t->codes_stride;
  d->sf_stride = t->sf_stride;
  d->ids_stride = t->ids_stride;
  d->weights_stride = t->weights_stride;
  d->scale_stride = t->scale_stride;
  d->num_tokens = t->num_tokens;
  d->topk = t->topk;
  d->k = t->k;
  d->epoch = t->epoch;
  d->parity_bytes = t->parity_bytes;
  if ((t->ids_stride & 3) || (t->weights_stride & 3) || (t->scale_stride & 3) ||
      !aligned4(t->ids) || !aligned4(t->weights) || !aligned4(t->scale))
    return set_error(FGG_EALIGN, "ids, weights and scale (and their strides) must be 4-byte aligned");
  return FGG_OK;
}

// 16-byte rows when every row start is 16-byte aligned, 4-byte otherwise.
bool rows_vec16(const MoeTok& t) {
  return aligned16(t.codes) && aligned16(t.sf) && t.codes_stride % 16 == 0 &&
         t.sf_stride % 16 == 0 && (t.k / 16) % 16 == 0;
}
bool rows_vec4(const MoeTok& t) {
  return aligned4(t.codes) && aligned4(t.sf) && t.codes_stride % 4 == 0 && t.sf_stride % 4 == 0 &&
         (t.k / 16) % 4 == 0;
}


}  // namespace
}  // namespace fgg

using namespace fgg;

extern "C" {

size_t fgg_moe_record_bytes(int32_t k, int32_t topk) {
  if (k < 64 || k % 64 != 0 || topk < 1) return 0;
  return align_up(size_t(k) / 2 + size_t(k) / 16 + 8u * size_t(topk) + 4u, 16);
}

int fgg_moe_pack_tokens(const FggMoeTokens* tokens, void* records, void* stream) {
  MoeTok t;
  if (int rc = to_dev(tokens, &t)) return rc;
  if (t.num_tokens == 0) return FGG_OK;
  if (records == nullptr || t.codes == nullptr || t.sf == nullptr)
    return set_error(FGG_EINVAL, "records / codes / sf is null");
  const size_t rb = fgg_moe_record_bytes(t.k, t.topk);
  if (!aligned16(records)) return set_error(FGG_EALIGN, "records must be 16-byte aligned");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const unsigned grid = unsigned((int64_t(t.num_tokens) + 7) / 8);  // 8 warps = 8 records a block
  if (rows_vec16(t))
    moe_pack_kernel<true><<<grid, 256, 0, s>>>(t, static_cast<uint8_t*>(records), int64_t(rb));
  else if (rows_vec4(t))
    moe_pack_kernel<false><<<grid, 256, 0, s>>>(t, static_cast<uint8_t*>(records), int64_t(rb));
  else
    return set_error(FGG_EALIGN, "token rows must start on 4-byte boundaries");
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

int fgg_moe_records_view(const void* records, int32_t num_tokens, int32_t k, int32_t topk,
                         FggMoeTokens* out) {
  if (out == nullptr) return set_error(FGG_EINVAL, "out is null");
  const size_t rb = fgg_moe_record_bytes(k, topk);
  if (rb == 0 || num_tokens < 0) return set_error(FGG_EBADSHAPE, "bad record geometry");
  const uint8_t* r = static_cast<const uint8_t*>(records);
  const size_t kh = size_t(k) / 2, ks = size_t(k) / 16;
  out->num_tokens = num_tokens;
  out->topk = topk;
  out->k = k;
  out->codes = r;
  out->sf = r + kh;
  out->ids = reinterpret_cast<const int32_t*>(r + kh + ks);
  out->weights = reinterpret_cast<const float*>(r + kh + ks + 4 * size_t(topk));
  out->scale = reinterpret_cast<const float*>(r + kh + ks + 8 * size_t(topk));
  out->codes_stride = out->sf_stride = out->ids_stride = out->weights_stride =
      out->scale_stride = int64_t(rb);
  out->epoch = nullptr;
  out->parity_bytes = 0;
  return FGG_OK;
}

}  // extern "C"

namespace fgg {
namespace {

int to_peers(const FggMoePeers* p, int64_t rb, PeerDev* x) {
  if (p == nullptr) return set_error(FGG_EINVAL, "peers is null");
  if (p->world < 1 || p->world > kPeersMax || p->rank < 0 || p->rank >= p->world ||
      p->capacity < 1 || p->n <= 0 || p->n % 8 != 0)
    return set_error(FGG_EBADSHAPE, "need 1 <= world <= %d, 0 <= rank < world, capacity >= 1, "
                                    "n a positive multiple of 8", kPeersMax);
  if (p->epoch == nullptr || p->counters == nullptr || p->status == nullptr ||
      p->owner == nullptr || p->routes == nullptr)
    return set_error(FGG_EINVAL, "epoch / counters / status / owner / routes is null");
  if (p->num_experts < 1) return set_error(FGG_EBADSHAPE, "num_experts must be positive");
  memset(x, 0, sizeof(*x));
  x->world = p->world;
  x->rank = p->rank;
  x->capacity = p->capacity;
  x->n = p->n;
  x->epoch = p->epoch;
  x->counters = p->counters;
  x->status = p->status;
  for (int s = 0; s < p->world; ++s) {
    if (p->gathered[s] == nullptr || p->recv[s] == nullptr || p->flags[s] == nullptr)
      return set_error(FGG_EINVAL, "rank %d's buffers are null", s);
    if (!aligned16(p->gathered[s]) || !aligned16(p->recv[s]) ||
        (reinterpret_cast<uintptr_t>(p->flags[s]) & 7u))
      return set_error(FGG_EALIGN, "rank %d's buffers are misaligned", s);
    x->gathered[s] = static_cast<uint8_t*>(p->gathered[s]);
    x->recv[s] = static_cast<uint8_t*>(p->recv[s]);
    x->flags[s] = static_cast<unsigned long long*>(p->flags[s]);
  }
  if (p->wait_ms < 0) return set_error(FGG_EINVAL, "wait_ms is negative");
  x->wait_ns = uint64_t(p->wait_ms > 0 ? p->wait_ms : kPeerWaitDefaultMs) * 1000000ull;
  x->owner = p->owner;
  x->num_experts = p->num_experts;
  x->routes = p->routes;
  x->rb = rb;
  x->gathered_half = int64_t(p->world) * p->capacity * rb;
  return FGG_OK;
}

}  // namespace
}  // namespace fgg

extern "C" {

int fgg_moe_dispatch_peers(const FggMoeTokens* tokens, const FggMoePeers* peers, void* stream) {
  MoeTok t;
  if (int rc = to_dev(tokens, &t)) return rc;
  if (t.epoch != nullptr) return set_error(FGG_EINVAL, "the dispatched tokens must be a plain view");
  const size_t rb = fgg_moe_record_bytes(t.k, t.topk);
  PeerDev x;
  if (int rc = to_peers(peers, int64_t(rb), &x)) return rc;
  if (t.num_tokens > x.capacity)
    return set_error(FGG_EBADSHAPE, "%d tokens exceed the capacity %d", t.num_tokens, x.capacity);
  if (t.num_tokens > 0 && (t.codes == nullptr || t.sf == nullptr))
    return set_error(FGG_EINVAL, "codes / sf is null");
  DeviceInfo dev;
  if (int rc = current_device(&dev)) return rc;
  // 8 warps a block, a warp per (token slot, destination rank)
  const int grid = int(std::min<int64_t>((int64_t(x.capacity) * x.world + 7) / 8,
                                         int64_t(dev.sm_count) * 8));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (rows_vec16(t) || t.num_tokens == 0)
    moe_dispatch_peers_kernel<true><<<grid, 256, 0, s>>>(t, x);
  else if (rows_vec4(t))
    moe_dispatch_peers_kernel<false><<<grid, 256, 0, s>>>(t, x);
  else
    return set_error(FGG_EALIGN, "token rows must start on 4-byte boundaries");
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

int fgg_moe_wait_peers(const FggMoePeers* peers, int32_t kind, void* stream) {
  PeerDev x;
  if (int rc = to_peers(peers, 0, &x)) return rc;
  if (kind != 0 && kind != 1) return set_error(FGG_EINVAL, "kind must be 0 (dispatch) or 1 (combine)");
  moe_wait_peers_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(x, kind);
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

int fgg_moe_reduce_peers(const void* rows, int32_t num_rows, const int32_t* route_row,
                         const FggMoeTokens* tokens, const FggMoePeers* peers, int* bad,
                         void* stream) {
  MoeTok t;
  if (int rc = to_dev(tokens, &t)) return rc;
  PeerDev x;
  if (int rc = to_peers(peers, 0, &x)) return rc;
  if (int64_t(t.num_tokens) != int64_t(x.world) * x.capacity)
    return set_error(FGG_EBADSHAPE, "the tokens must be the world * capacity gathered slots");
  if (num_rows < 0) return set_error(FGG_EINVAL, "num_rows is negative");
  if (route_row == nullptr || bad == nullptr || (num_rows > 0 && rows == nullptr))
    return set_error(FGG_EINVAL, "null pointer");
  if (!aligned16(rows)) return set_error(FGG_EALIGN, "rows must be 16-byte aligned");
  const dim3 grid(unsigned(t.num_tokens), unsigned((x.n / 8 + 255) / 256));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // the partial rows stay in this rank's memory; their tokens' ranks read them
  FGG_CUDA_CHECK(launch_pdl(moe_reduce_kernel, grid, dim3(256), 0, s, t,
                            static_cast<const __nv_bfloat16*>(rows), num_rows, route_row, x.n,
                            reinterpret_cast<__nv_bfloat16*>(x.recv[x.rank]), bad, 1));
  moe_signal_peers_kernel<<<1, 32, 0, s>>>(x, 1);
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

int fgg_moe_sum_peers(const FggMoePeers* peers, int32_t tokens, void* out, void* stream) {
  PeerDev x;
  if (int rc = to_peers(peers, 0, &x)) return rc;
  if (tokens < 0 || tokens > x.capacity)
    return set_error(FGG_EBADSHAPE, "tokens=%d outside [0, capacity=%d]", tokens, x.capacity);
  if (out == nullptr && tokens > 0) return set_error(FGG_EINVAL, "out is null");
  if (tokens > 0 && !aligned16(out)) return set_error(FGG_EALIGN, "out must be 16-byte aligned");
  // at least one block even for zero tokens: the last block advances the epoch
  const dim3 grid(unsigned(std::max(tokens, 1)), unsigned((x.n / 8 + 255) / 256));
  FGG_CUDA_CHECK(launch_pdl(moe_sum_peers_kernel, grid, dim3(256), 0,
                            reinterpret_cast<cudaStream_t>(stream), x, tokens,
                            static_cast<__nv_bfloat16*>(out)));
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

int fgg_moe_expand(const FggMoeTokens* tokens, const int32_t* owner, const int32_t* slot,
                   int32_t num_experts, int32_t rank, int32_t local, int32_t max_rows,
                   int32_t* counts, int32_t* offsets, int32_t* route_row, int32_t* src_token,
                   float* row_scale, void* out_codes, void* out_sf, int* bad, void* stream) {
  MoeTok t;
  if (int rc = to_dev(tokens, &t)) return rc;
  if (num_experts < 1 || local < 1 || local > kExpandMaxLocal || rank < 0 || max_rows < 0)
    return set_error(FGG_EBADSHAPE, "need num_experts >= 1, 1 <= local <= %d, rank >= 0",
                     kExpandMaxLocal);
  const int64_t routes = int64_t(t.num_tokens) * t.topk;
  if (routes > INT32_MAX) return set_error(FGG_EBADSHAPE, "too many routes");
  if (owner == nullptr || slot == nullptr || counts == nullptr || offsets == nullptr ||
      bad == nullptr || (routes > 0 && route_row == nullptr) ||
      (max_rows > 0 && (src_token == nullptr || row_scale == nullptr || out_codes == nullptr ||
                        out_sf == nullptr)))
    return set_error(FGG_EINVAL, "null pointer");
  if (routes > 0 && (t.codes == nullptr || t.sf == nullptr))
    return set_error(FGG_EINVAL, "codes / sf is null");
  const bool v16 = rows_vec16(t) && aligned16(out_codes) && aligned16(out_sf);
  const bool v4 = rows_vec4(t) && aligned4(out_codes) && aligned4(out_sf);
  if (routes > 0 && !v16 && !v4)
    return set_error(FGG_EALIGN, "token rows must start on 4-byte boundaries");
  DeviceInfo dev;
  if (int rc = current_device(&dev)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // counts[0, local) and the cursors counts[local, 2 local)
  FGG_CUDA_CHECK(cudaMemsetAsync(counts, 0, 2 * size_t(local) * sizeof(int32_t), s));
  const int count_grid = int(std::min<int64_t>((routes + 255) / 256, int64_t(dev.sm_count) * 2));
  FGG_CUDA_CHECK(launch_pdl(moe_expand_count_kernel, dim3(std::max(count_grid, 1)), dim3(256), 0,
                            s, t, owner, slot, num_experts, rank, local, counts, bad));
  const int place_grid = int(std::min<int64_t>((routes + 7) / 8, int64_t(dev.sm_count) * 8));
  auto* oc = static_cast<uint8_t*>(out_codes);
  auto* of = static_cast<uint8_t*>(out_sf);
  if (v16)
    FGG_CUDA_CHECK(launch_pdl(moe_expand_place_kernel<true>, dim3(std::max(place_grid, 1)),
                              dim3(256), 0, s, t, owner, slot, num_experts, rank, local, max_rows,
                              counts, counts + local, offsets, route_row, src_token, row_scale, oc,
                              of, bad));
  else
    FGG_CUDA_CHECK(launch_pdl(moe_expand_place_kernel<false>, dim3(std::max(place_grid, 1)),
                              dim3(256), 0, s, t, owner, slot, num_experts, rank, local, max_rows,
                              counts, counts + local, offsets, route_row, src_token, row_scale, oc,
                              of, bad));
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

int fgg_moe_reduce(const void* rows, int32_t num_rows, const int32_t* route_row,
                   const FggMoeTokens* tokens, int32_t n, void* out, int* bad, void* stream) {
  MoeTok t;
  if (int rc = to_dev(tokens, &t)) return rc;
  if (n <= 0 || n % 8 != 0 || num_rows < 0)
    return set_error(FGG_EBADSHAPE, "n must be a positive multiple of 8");
  if (t.num_tokens == 0) return FGG_OK;
  if (route_row == nullptr || out == nullptr || bad == nullptr || (num_rows > 0 && rows == nullptr))
    return set_error(FGG_EINVAL, "null pointer");
  if (!aligned16(rows) || !aligned16(out))
    return set_error(FGG_EALIGN, "rows and out must be 16-byte aligned");
  const dim3 grid(unsigned(t.num_tokens), unsigned((n / 8 + 255) / 256));
  FGG_CUDA_CHECK(launch_pdl(moe_reduce_kernel, grid, dim3(256), 0,
                            reinterpret_cast<cudaStream_t>(stream), t,
                            static_cast<const __nv_bfloat16*>(rows), num_rows, route_row, n,
                            static_cast<__nv_bfloat16*>(out), bad, 0));
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

int fgg_moe_sum_partials(const void* parts, int32_t world, int32_t per_source, int32_t tokens,
                         int32_t n, void* out, void* stream) {
  if (world < 1 || tokens < 0 || per_source < tokens || n <= 0 || n % 8 != 0)
    return set_error(FGG_EBADSHAPE, "need world >= 1, 0 <= tokens <= per_source, n a positive "
                                    "multiple of 8");
  if (tokens == 0) return FGG_OK;
  if (parts == nullptr || out == nullptr) return set_error(FGG_EINVAL, "null pointer");
  if (!aligned16(parts) || !aligned16(out))
    return set_error(FGG_EALIGN, "parts and out must be 16-byte aligned");
  const dim3 grid(unsigned(tokens), unsigned((n / 8 + 255) / 256));
  FGG_CUDA_CHECK(launch_pdl(moe_sum_parts_kernel, grid, dim3(256), 0,
                            reinterpret_cast<cudaStream_t>(stream),
                            static_cast<const __nv_bfloat16*>(parts), world, per_source, tokens, n,
                            static_cast<__nv_bfloat16*>(out)));
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

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
