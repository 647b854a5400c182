// fgg_nvfp4.cu - NVFP4 x NVFP4 grouped GEMM entry points (per-group lists).
//
// Per call:
//   1. nvfp4_prepare_kernel  per-group TMA descriptors for the token tensors
//                            (edited on the device from one host-encoded
//                            template), the token scales repacked into 512-byte
//                            SF atoms, the flat tile list, status reset.
//   2. fgg_gemm_kernel<NVFP4 cfg>  (fgg_engine.cuh).
// Weights are packed once by nvfp4_pack_weights_kernel (descriptors + SF
// atoms) and cached by the caller, as kernel.py:2743-2786 caches its repack.
#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>

#include "fgg_engine.cuh"
#include "fgg_host.cuh"

namespace fgg {

// activation bytes up to which the tile list runs weight-tile-major over all
// groups (a quarter of the 126 MB L2: the weights in flight need the rest)
constexpr int64_t kAcrossGroupsMaxBytes = 32ll << 20;

// ------------------------------------------------------- prepare kernels
// The per-group arrays travel as kernel parameters; CAP groups of room (a
// small instance for the common few-group call keeps the launch light).
template <int CAP>
struct PrepParams {
  CUtensorMap tmpl;  // token descriptor template (group 0's geometry)
  const uint8_t* a[CAP];
  const uint8_t* a_sf[CAP];
  int32_t m[CAP];
  int32_t xtile_begin[CAP + 1];
  int32_t tile_begin[CAP + 1];
  int32_t out_row[CAP];
  int32_t wgroup[CAP];  // weight group of each problem group
  CUtensorMap* tmap_out;
  GroupInfo* ginfo_out;
  uint32_t* tiles_out;
  uint8_t* sfx_out;
  int* status;
  int32_t g, k, bn, ch, nk64p, nt, num_tiles, xt_total;
  int32_t blocks_tmap, blocks_tiles;
  int32_t across_groups;
  int32_t sf_vec;  // 1: K % 256 == 0 and every a_sf[g] 16-byte aligned (vector repack)  // tile order: 1 weight-tile-major over all groups, 0 group-major
};

// Group whose tiles (its token tiles x nt weight tiles, group-major) hold tile t.
__device__ __forceinline__ int find_group_tiles(const int32_t* begin, int g_count, int t, int nt) {
  int lo = 0, hi = g_count;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (begin[mid] * nt <= t)
      lo = mid;
    else
      hi = mid;
  }
  return lo;
}

__device__ __forceinline__ int find_group(const int32_t* begin, int g_count, int x) {
  int lo = 0, hi = g_count;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (begin[mid] <= x)
      lo = mid;
    else
      hi = mid;
  }
  return lo;
}

template <int CAP>
__global__ void __launch_bounds__(256)
    nvfp4_prepare_kernel(const __grid_constant__ PrepParams<CAP> p) {
  // every block is resident once it gets here: the GEMM grid behind this one
  // may launch now (it waits for this grid's results before reading them)
  griddep_launch_dependents();
  // launched early behind the previous GEMM: touch no memory before it is done
  griddep_wait();
  __shared__ alignas(128) CUtensorMap smap[8];
  __shared__ int32_t sbegin[CAP + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int blk = blockIdx.x;
  if (blk < p.blocks_tmap) {
    if (blk == 0 && threadIdx.x == 0) {
      p.status[0] = 0;
      p.status[1] = 0;
      p.status[2] = 0;
    }
    const int g = blk * 8 + warp;
    if (g < p.g) {
      const uint32_t* src = reinterpret_cast<const uint32_t*>(&p.tmpl);
      reinterpret_cast<uint32_t*>(&smap[warp])[lane] = src[lane];
      __syncwarp();
      if (lane == 0) {
        tmap_replace_address(smem_u32(&smap[warp]), reinterpret_cast<uint64_t>(p.a[g]));
        tmap_replace_dim1(smem_u32(&smap[warp]), max(p.m[g], 1));
        GroupInfo gi;
        gi.m = p.m[g];
        gi.out_row = p.out_row[g];
        gi.xtile_begin = p.xtile_begin[g];
        gi.wgroup = p.wgroup[g];
        p.ginfo_out[g] = gi;
      }
      __syncwarp();
      tmap_publish(p.tmap_out + g, smem_u32(&smap[warp]));
    }
    return;
  }
  blk -= p.blocks_tmap;
  if (blk < p.blocks_tiles) {
    if (p.across_groups) {
      // Weight-tile-major over all groups: tile t pairs weight tile
      // t / xt_total with token tile t % xt_total of the groups' concatenated
      // token tiles.  The tiles running at any moment span every group, so
      // the groups whose weights serve one token tile (read from DRAM for it
      // alone) spread over the whole kernel instead of gathering at its end.
      for (int i = threadIdx.x; i <= p.g; i += blockDim.x) sbegin[i] = p.xtile_begin[i];
      __syncthreads();
      const int t = blk * blockDim.x + threadIdx.x;
      if (t < p.num_tiles) {
        const int nti = t / p.xt_total;
        const int X = t - nti * p.xt_total;
        const int g = find_group(sbegin, p.g, X);
        p.tiles_out[t] = pack_tile(g, nti, X - sbegin[g]);
      }
    } else {
      // group-major: each group's weight tiles in turn, its token tiles fastest
      for (int i = threadIdx.x; i <= p.g; i += blockDim.x) sbegin[i] = p.tile_begin[i];
      __syncthreads();
      const int t = blk * blockDim.x + threadIdx.x;
      if (t < p.num_tiles) {
        const int g = find_group(sbegin, p.g, t);
        const int local = t - sbegin[g];
        const int xts = p.xtile_begin[g + 1] - p.xtile_begin[g];
        p.tiles_out[t] = pack_tile(g, local / xts, local % xts);
      }
    }
    return;
  }
  blk -= p.blocks_tiles;
  // Token scales -> SF atoms:
  //   atom byte (r % 32) * 16 + (r / 32) * 4 + b  <-  sf[row r][4 j + b]
  for (int i = threadIdx.x; i <= p.g; i += blockDim.x) sbegin[i] = p.xtile_begin[i];
  __syncthreads();
  if (p.sf_vec) {
    // K % 256 == 0 and 16-byte aligned scale rows: one thread loads 16 bytes
    // (the scales of one K step of 4 MMAs) from each of its 4 rows and writes
    // the 16-byte atom row of every MMA of that K step.
    const int64_t quad = int64_t(blk) * blockDim.x + threadIdx.x;
    const int nk256 = p.nk64p / 4;
    const int64_t quads_per_xt = int64_t(nk256) * p.ch * 32;
    if (quad >= int64_t(p.xt_total) * quads_per_xt) return;
    const int X = int(quad / quads_per_xt);
    const int rem = int(quad - int64_t(X) * quads_per_xt);
    const int s4 = rem / (p.ch * 32);
    const int c = (rem / 32) % p.ch;
    const int r0 = rem & 31;
    const int g = find_group(sbegin, p.g, X);
    const int xt = X - sbegin[g];
    const int kq = p.k / 16;
    uint4 v[4];
#pragma unroll
    for (int r1 = 0; r1 < 4; ++r1) {
      const int rr = c * 128 + r1 * 32 + r0;
      const int row = xt * p.bn + rr;
      v[r1] = make_uint4(0u, 0u, 0u, 0u);
      if (rr < p.bn && row < p.m[g])
        v[r1] = __ldg(reinterpret_cast<const uint4*>(p.a_sf[g] + size_t(row) * kq + 16 * s4));
    }
    uint8_t* dst = p.sfx_out + ((size_t(X) * p.nk64p + 4 * s4) * p.ch + c) * 512u + size_t(r0) * 16u;
    const size_t jstride = size_t(p.ch) * 512u;
    *reinterpret_cast<uint4*>(dst) = make_uint4(v[0].x, v[1].x, v[2].x, v[3].x);
    *reinterpret_cast<uint4*>(dst + jstride) = make_uint4(v[0].y, v[1].y, v[2].y, v[3].y);
    *reinterpret_cast<uint4*>(dst + 2 * jstride) = make_uint4(v[0].z, v[1].z, v[2].z, v[3].z);
    *reinterpret_cast<uint4*>(dst + 3 * jstride) = make_uint4(v[0].w, v[1].w, v[2].w, v[3].w);
    return;
  }
  // general case: one thread writes one 16-byte atom row
  const int64_t line = int64_t(blk) * blockDim.x + threadIdx.x;
  const int64_t lines_per_xt = int64_t(p.nk64p) * p.ch * 32;
  if (line >= int64_t(p.xt_total) * lines_per_xt) return;
  const int X = int(line / lines_per_xt);
  const int rem = int(line - int64_t(X) * lines_per_xt);
  const int j = rem / (p.ch * 32);
  const int c = (rem / 32) % p.ch;
  const int r0 = rem & 31;
  const int g = find_group(sbegin, p.g, X);
  const int xt = X - sbegin[g];
  const int kq = p.k / 16;
  uint32_t v[4];
#pragma unroll
  for (int r1 = 0; r1 < 4; ++r1) {
    const int rr = c * 128 + r1 * 32 + r0;
    const int row = xt * p.bn + rr;
    v[r1] = 0u;
    if (rr < p.bn && row < p.m[g] && 4 * j < kq)
      v[r1] = __ldg(reinterpret_cast<const uint32_t*>(p.a_sf[g] + size_t(row) * kq + 4 * j));
  }
  *reinterpret_cast<uint4*>(p.sfx_out + ((size_t(X) * p.nk64p + j) * p.ch + c) * 512u +
                            size_t(r0) * 16u) = make_uint4(v[0], v[1], v[2], v[3]);
}

// ------------------------------------------- prepare, device group offsets
// The contiguous-rows form: every group's token rows lie in one buffer, group
// g owning rows [offsets[g], offsets[g+1]) with the offsets in device memory
// (written by an earlier kernel, e.g. an expert-parallel dispatch plan), so
// the host never learns the group sizes.  Every block of this kernel rebuilds
// the per-group token-tile prefix from the offsets in shared memory; block 0
// also writes the status words, the tile count and the GroupInfo table.
constexpr int kStatusBadOffsets = 0x203;  // offsets decreasing or past max_rows

struct RowsPrepParams {
  const int32_t* offsets;  // [G + 1] device
  const int32_t* b_index;  // [G] device or null
  const uint8_t* a_sf;     // [max_rows, K/16]
  GroupInfo* ginfo_out;
  uint32_t* tiles_out;
  uint8_t* sfx_out;
  int* status;             // [0] status [1] tile counter [2] finished CTAs [3] tile count
  int32_t g, wg, k, bn, ch, nk64p, nt, max_rows;
  int32_t tile_cap, xt_cap;  // room in tiles_out / token tiles in sfx_out
  int32_t blocks_tiles;
  int32_t sf_vec;     // K % 256 == 0 and a_sf 16-byte aligned
  int32_t decode;     // decode tiles: never the across-groups order
};

// Shared-memory prefix of the token tiles per group: begin[g] for g <= G.
// Returns the total, or -1 when the offsets are malformed.
__device__ int rows_tile_prefix(const RowsPrepParams& p, int32_t* begin, int32_t* off) {
  __shared__ int s_bad;
  __shared__ int32_t s_warp[8];
  if (threadIdx.x == 0) s_bad = 0;
  for (int i = threadIdx.x; i <= p.g; i += blockDim.x) off[i] = __ldg(p.offsets + i);
  __syncthreads();
  // each thread sums the tiles of a contiguous run of groups
  const int per = (p.g + blockDim.x - 1) / blockDim.x;
  const int g0 = threadIdx.x * per, g1 = min(p.g, g0 + per);
  int run = 0;
  for (int g = g0; g < g1; ++g) {
    const int m = off[g + 1] - off[g];
    if (m < 0 || off[g] < 0 || off[g + 1] > p.max_rows) s_bad = 1;
    run += m > 0 ? (m + p.bn - 1) / p.bn : 0;
  }
  // block-wide exclusive scan of the runs
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += y;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  int wbase = 0;
  for (int w = 0; w < warp; ++w) wbase += s_warp[w];
  int acc = wbase + incl - run;
  for (int g = g0; g < g1; ++g) {
    begin[g] = acc;
    const int m = off[g + 1] - off[g];
    acc += m > 0 ? (m + p.bn - 1) / p.bn : 0;
  }
  if (threadIdx.x == blockDim.x - 1) begin[p.g] = wbase + incl;
  __syncthreads();
  if (s_bad) return -1;
  return begin[p.g];
}

__global__ void __launch_bounds__(256)
    nvfp4_prepare_rows_kernel(const __grid_constant__ RowsPrepParams p) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ int32_t sbegin[FGG_MAX_GROUPS + 1];
  __shared__ int32_t soff[FGG_MAX_GROUPS + 1];
  const int xt_total = rows_tile_prefix(p, sbegin, soff);
  const bool bad = xt_total < 0 || xt_total > p.xt_cap;
  const int num_tiles = bad ? 0 : xt_total * p.nt;
  int blk = blockIdx.x;
  if (blk == 0) {
    if (threadIdx.x == 0) {
      p.status[0] = bad ? kStatusBadOffsets : 0;
      p.status[1] = 0;
      p.status[2] = 0;
      p.status[3] = num_tiles;
    }
    for (int g = threadIdx.x; g < p.g; g += blockDim.x) {
      GroupInfo gi;
      gi.m = bad ? 0 : soff[g + 1] - soff[g];
      gi.out_row = soff[g];
      gi.xtile_begin = bad ? 0 : sbegin[g];
      int wg = p.b_index != nullptr ? __ldg(p.b_index + g) : g;
      gi.wgroup = wg;
      p.ginfo_out[g] = gi;
    }
    return;
  }
  if (bad) return;
  blk -= 1;
  if (blk < p.blocks_tiles) {
    const int t = blk * blockDim.x + threadIdx.x;
    if (t >= num_tiles) return;
    const bool across = !p.decode && p.g > 1 &&
                        int64_t(soff[p.g]) * (p.k / 2 + p.k / 16) <= kAcrossGroupsMaxBytes;
    if (across) {
      const int nti = t / xt_total;
      const int X = t - nti * xt_total;
      const int g = find_group(sbegin, p.g, X);
      p.tiles_out[t] = pack_tile(g, nti, X - sbegin[g]);
    } else {
      // group-major: a group's tiles are its token tiles x NT weight tiles
      const int X0 = find_group_tiles(sbegin, p.g, t, p.nt);
      const int g = X0;
      const int local = t - sbegin[g] * p.nt;
      const int xts = sbegin[g + 1] - sbegin[g];
      p.tiles_out[t] = pack_tile(g, local / xts, local % xts);
    }
    return;
  }
  blk -= p.blocks_tiles;
  const int kq = p.k / 16;
  if (p.sf_vec) {
    const int64_t quad = int64_t(blk) * blockDim.x + threadIdx.x;
    const int nk256 = p.nk64p / 4;
    const int64_t quads_per_xt = int64_t(nk256) * p.ch * 32;
    if (quad >= int64_t(xt_total) * quads_per_xt) return;
    const int X = int(quad / quads_per_xt);
    const int rem = int(quad - int64_t(X) * quads_per_xt);
    const int s4 = rem / (p.ch * 32);
    const int c = (rem / 32) % p.ch;
    const int r0 = rem & 31;
    const int g = find_group(sbegin, p.g, X);
    const int xt = X - sbegin[g];
    const int m = soff[g + 1] - soff[g];
    uint4 v[4];
#pragma unroll
    for (int r1 = 0; r1 < 4; ++r1) {
      const int rr = c * 128 + r1 * 32 + r0;
      const int row = xt * p.bn + rr;
      v[r1] = make_uint4(0u, 0u, 0u, 0u);
      if (rr < p.bn && row < m)
        v[r1] = __ldg(reinterpret_cast<const uint4*>(p.a_sf + size_t(soff[g] + row) * kq + 16 * s4));
    }
    uint8_t* dst = p.sfx_out + ((size_t(X) * p.nk64p + 4 * s4) * p.ch + c) * 512u + size_t(r0) * 16u;
    const size_t jstride = size_t(p.ch) * 512u;
    *reinterpret_cast<uint4*>(dst) = make_uint4(v[0].x, v[1].x, v[2].x, v[3].x);
    *reinterpret_cast<uint4*>(dst + jstride) = make_uint4(v[0].y, v[1].y, v[2].y, v[3].y);
    *reinterpret_cast<uint4*>(dst + 2 * jstride) = make_uint4(v[0].z, v[1].z, v[2].z, v[3].z);
    *reinterpret_cast<uint4*>(dst + 3 * jstride) = make_uint4(v[0].w, v[1].w, v[2].w, v[3].w);
    return;
  }
  const int64_t line = int64_t(blk) * blockDim.x + threadIdx.x;
  const int64_t lines_per_xt = int64_t(p.nk64p) * p.ch * 32;
  if (line >= int64_t(xt_total) * lines_per_xt) return;
  const int X = int(line / lines_per_xt);
  const int rem = int(line - int64_t(X) * lines_per_xt);
  const int j = rem / (p.ch * 32);
  const int c = (rem / 32) % p.ch;
  const int r0 = rem & 31;
  const int g = find_group(sbegin, p.g, X);
  const int xt = X - sbegin[g];
  const int m = soff[g + 1] - soff[g];
  uint32_t v[4];
#pragma unroll
  for (int r1 = 0; r1 < 4; ++r1) {
    const int rr = c * 128 + r1 * 32 + r0;
    const int row = xt * p.bn + rr;
    v[r1] = 0u;
    if (rr < p.bn && row < m && 4 * j < kq)
      v[r1] = __ldg(reinterpret_cast<const uint32_t*>(p.a_sf + size_t(soff[g] + row) * kq + 4 * j));
  }
  *reinterpret_cast<uint4*>(p.sfx_out + ((size_t(X) * p.nk64p + j) * p.ch + c) * 512u +
                            size_t(r0) * 16u) = make_uint4(v[0], v[1], v[2], v[3]);
}

struct PackParams {
  CUtensorMap tmpl;
  const uint8_t* b[FGG_MAX_GROUPS];
  const uint8_t* b_sf[FGG_MAX_GROUPS];
  PackHeader* header;
  CUtensorMap* tmap_out;
  uint8_t* sfw_out;
  int32_t g, n, k, nk64p, nt;
  int32_t blocks_tmap;
};

__global__ void __launch_bounds__(256) nvfp4_pack_weights_kernel(const __grid_constant__ PackParams p) {
  __shared__ alignas(128) CUtensorMap smap[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int blk = blockIdx.x;
  if (blk < p.blocks_tmap) {
    if (blk == 0 && threadIdx.x == 0) {
      PackHeader h;
      h.magic = kPackMagic;
      h.g = p.g;
      h.n = p.n;
      h.k = p.k;
      *p.header = h;
    }
    const int g = blk * 8 + warp;
    if (g < p.g) {
      reinterpret_cast<uint32_t*>(&smap[warp])[lane] =
          reinterpret_cast<const uint32_t*>(&p.tmpl)[lane];
      __syncwarp();
      if (lane == 0) tmap_replace_address(smem_u32(&smap[warp]), reinterpret_cast<uint64_t>(p.b[g]));
      __syncwarp();
      tmap_publish(p.tmap_out + g, smem_u32(&smap[warp]));
    }
    return;
  }
  blk -= p.blocks_tmap;
  const int64_t line = int64_t(blk) * blockDim.x + threadIdx.x;
  const int64_t total = int64_t(p.g) * p.nt * p.nk64p * 32;
  if (line >= total) return;
  const int r0 = int(line & 31);
  int64_t rest = line >> 5;
  const int j = int(rest % p.nk64p);
  rest /= p.nk64p;
  const int nt = int(rest % p.nt);
  const int g = int(rest / p.nt);
  const int kq = p.k / 16;
  uint32_t v[4];
#pragma unroll
  for (int r1 = 0; r1 < 4; ++r1) {
    const int row = nt * 128 + r1 * 32 + r0;
    v[r1] = (4 * j < kq)
                ? __ldg(reinterpret_cast<const uint32_t*>(p.b_sf[g] + size_t(row) * kq + 4 * j))
                : 0u;
  }
  uint4* dst = reinterpret_cast<uint4*>(p.sfw_out + ((size_t(g) * p.nt + nt) * p.nk64p + j) * 512u +
                                        size_t(r0) * 16u);
  *dst = make_uint4(v[0], v[1], v[2], v[3]);
}

// ------------------------------------------------------------ host side
using CfgPrefill = EngineCfg<false, 224, 4>;   // one CTA per tile (N % 256 != 0)
using CfgDecode = EngineCfg<false, 16, 4, 2>;  // every group has M <= 16; 2 K steps per stage
using CfgPair = PairCfg<false, 6>;             // CTA pairs, 256 x 224 tiles

struct PackLayout {
  size_t header, tmaps, sfw, total;
};
static PackLayout pack_layout(int g, int n, int k) {
  const int nk64p = ((k / 64) + 3) / 4 * 4;
  Carver cv;
  PackLayout L;
  L.header = cv.take(sizeof(PackHeader), 256);
  L.tmaps = cv.take(size_t(g) * sizeof(CUtensorMap), 128);
  L.sfw = cv.take(size_t(g) * (n / 128) * nk64p * 512, 256);
  L.total = cv.off;
  return L;
}


struct WsLayout {
  int bn = 0, ch = 0, stages = 0;
  bool pair = false;
  int box_rows = 0;  // token rows per TMA box (a pair CTA loads half a tile)
  int nk64p = 0, nk256 = 0, nt = 0, nt128 = 0;
  int num_tiles = 0, xt_total = 0;
  // per-group bookkeeping in fixed arrays: planning a call touches no host heap
  int32_t xtile_begin[FGG_MAX_GROUPS + 1];
  int32_t tile_begin[FGG_MAX_GROUPS + 1];
  int32_t out_row[FGG_MAX_GROUPS];
  int wg = 0;  // weight groups the problem groups index into
  // Tile order.  Weight-tile-major over all groups re-reads every token tile
  // once per weight tile, which pays while the activations stay in L2 (they
  // are re-read from there) and spreads the single-use weights of small groups
  // over the kernel; with more activation bytes than kAcrossGroupsMaxBytes the
  // order stays group-major, so a group's token tiles share each weight tile
  // while it is hot.  Decode tiles stream their weights once in either order.
  bool across_groups = false;
  size_t status = 0, tmaps = 0, ginfo = 0, tiles = 0, sfx = 0, total = 0;
};

static int plan(const FggNvfp4Problem* p, WsLayout* L) {
  if (p == nullptr) return set_error(FGG_EINVAL, "problem is null");
  const int G = p->num_groups;
  if (G < 1 || G > FGG_MAX_GROUPS)
    return set_error(FGG_EINVAL, "num_groups=%d outside [1, %d]", G, FGG_MAX_GROUPS);
  if (p->n <= 0 || p->n % 128 != 0)
    return set_error(FGG_EBADSHAPE, "N=%d must be a positive multiple of 128", p->n);
  if (p->k < 64 || p->k % 64 != 0)
    return set_error(FGG_EBADSHAPE, "K=%d must be a positive multiple of 64", p->k);
  if (p->m == nullptr) return set_error(FGG_EINVAL, "m (host problem sizes) is null");
  if (p->n / 128 > 2047) return set_error(FGG_EBADSHAPE, "N=%d too large", p->n);
  L->wg = G;
  if (p->b_index != nullptr) {
    // several problem groups may share one packed weight group (e.g. the
    // per-source chunks of one expert after an all-to-all dispatch)
    if (p->num_weight_groups < 1 || p->num_weight_groups > FGG_MAX_GROUPS)
      return set_error(FGG_EINVAL, "num_weight_groups=%d outside [1, %d]", p->num_weight_groups,
                       FGG_MAX_GROUPS);
    for (int g = 0; g < G; ++g)
      if (p->b_index[g] < 0 || p->b_index[g] >= p->num_weight_groups)
        return set_error(FGG_EINVAL, "b_index[%d]=%d outside [0, %d)", g, p->b_index[g],
                         p->num_weight_groups);
    L->wg = p->num_weight_groups;
  }
  int maxm = 0;
  for (int g = 0; g < G; ++g) {
    if (p->m[g] < 0) return set_error(FGG_EINVAL, "m[%d]=%d is negative", g, p->m[g]);
    maxm = std::max(maxm, p->m[g]);
  }
  const bool decode = maxm <= 16;
  L->pair = !decode && (p->n % 256 == 0);
  L->bn = decode ? CfgDecode::BN : CfgPrefill::BN;  // 224 for both the pair and single CTA
  L->ch = decode ? CfgDecode::CH : CfgPrefill::CH;
  L->stages = decode ? CfgDecode::STAGES : (L->pair ? CfgPair::STAGES : CfgPrefill::STAGES);
  L->box_rows = L->pair ? CfgPair::BNH : L->bn;
  L->nk256 = (p->k + 255) / 256;
  L->nk64p = 4 * L->nk256;
  L->nt128 = p->n / 128;
  L->nt = L->pair ? p->n / 256 : L->nt128;
  int64_t rows = 0, xts = 0, tiles = 0;
  for (int g = 0; g < G; ++g) {
    L->out_row[g] = int32_t(rows);
    L->xtile_begin[g] = int32_t(xts);
    L->tile_begin[g] = int32_t(tiles);
    const int64_t xt = (p->m[g] + L->bn - 1) / L->bn;
    if (xt > 2047) return set_error(FGG_EBADSHAPE, "m[%d]=%d too large", g, p->m[g]);
    rows += p->m[g];
    xts += xt;
    tiles += xt * L->nt;
  }
  if (rows > INT32_MAX || tiles > INT32_MAX) return set_error(FGG_EBADSHAPE, "problem too large");
  L->xtile_begin[G] = int32_t(xts);
  L->across_groups = !decode && G > 1 &&
                     rows * (p->k / 2 + p->k / 16) <= int64_t(kAcrossGroupsMaxBytes);
  L->tile_begin[G] = int32_t(tiles);
  L->num_tiles = int(tiles);
  L->xt_total = int(xts);
  Carver cv;
  L->status = cv.take(kStatusBytes, 256);
  L->tmaps = cv.take(size_t(G) * sizeof(CUtensorMap), 128);
  L->ginfo = cv.take(size_t(G) * sizeof(GroupInfo), 256);
  L->tiles = cv.take(size_t(std::max<int64_t>(tiles, 1)) * 4, 256);
  // token scales per (token tile, MMA): ch atoms of 512 B
  L->sfx = cv.take(size_t(std::max<int64_t>(xts, 1)) * L->nk64p * L->ch * 512, 256);
  L->total = cv.off;
  return FGG_OK;
}

}  // namespace fgg

using namespace fgg;

extern "C" {

size_t fgg_nvfp4_weight_pack_bytes(int32_t num_groups, int32_t n, int32_t k) {
  if (num_groups < 1 || n <= 0 || k <= 0) return 0;
  return pack_layout(num_groups, n, k).total;
}

int fgg_nvfp4_pack_weights(const FggNvfp4Weights* w, void* pack, size_t pack_bytes, void* stream) {
  if (w == nullptr || pack == nullptr) return set_error(FGG_EINVAL, "weights or pack is null");
  const int G = w->num_groups;
  if (G < 1 || G > FGG_MAX_GROUPS)
    return set_error(FGG_EINVAL, "num_groups=%d outside [1, %d]", G, FGG_MAX_GROUPS);
  if (w->n <= 0 || w->n % 128 != 0)
    return set_error(FGG_EBADSHAPE, "N=%d must be a positive multiple of 128", w->n);
  if (w->k < 64 || w->k % 64 != 0)
    return set_error(FGG_EBADSHAPE, "K=%d must be a positive multiple of 64", w->k);
  if (w->b == nullptr || w->b_sf == nullptr) return set_error(FGG_EINVAL, "b / b_sf arrays are null");
  for (int g = 0; g < G; ++g) {
    if (w->b[g] == nullptr || w->b_sf[g] == nullptr)
      return set_error(FGG_EINVAL, "group %d weight pointer is null", g);
    if (!aligned16(w->b[g])) return set_error(FGG_EALIGN, "b[%d] is not 16-byte aligned", g);
    if (!aligned4(w->b_sf[g])) return set_error(FGG_EALIGN, "b_sf[%d] is not 4-byte aligned", g);
  }
  if (!aligned16(pack)) return set_error(FGG_EALIGN, "pack is not 16-byte aligned");
  const PackLayout L = pack_layout(G, w->n, w->k);
  if (pack_bytes < L.total)
    return set_error(FGG_EWORKSPACE, "pack has %zu bytes, needs %zu", pack_bytes, L.total);
  DeviceInfo dev;
  if (int rc = current_device(&dev)) return rc;

  PackParams pp;
  memset(&pp, 0, sizeof(pp));
  if (int rc = encode_u8_2d(&pp.tmpl, w->b[0], uint64_t(w->k) / 2, uint64_t(w->n), 128, 128))
    return rc;
  for (int g = 0; g < G; ++g) {
    pp.b[g] = static_cast<const uint8_t*>(w->b[g]);
    pp.b_sf[g] = static_cast<const uint8_t*>(w->b_sf[g]);
  }
  uint8_t* base = static_cast<uint8_t*>(pack);
  pp.header = reinterpret_cast<PackHeader*>(base + L.header);
  pp.tmap_out = reinterpret_cast<CUtensorMap*>(base + L.tmaps);
  pp.sfw_out = base + L.sfw;
  pp.g = G;
  pp.n = w->n;
  pp.k = w->k;
  pp.nk64p = ((w->k / 64) + 3) / 4 * 4;
  pp.nt = w->n / 128;
  pp.blocks_tmap = (G + 7) / 8;
  const int64_t lines = int64_t(G) * pp.nt * pp.nk64p * 32;
  const int64_t blocks = pp.blocks_tmap + (lines + 255) / 256;
  if (blocks > INT32_MAX) return set_error(FGG_EBADSHAPE, "weights too large");
  nvfp4_pack_weights_kernel<<<int(blocks), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(pp);
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

size_t fgg_nvfp4_workspace_bytes(const FggNvfp4Problem* p) {
  WsLayout L;
  if (plan(p, &L) != FGG_OK) return 0;
  return L.total;
}

}  // extern "C"

namespace fgg {
namespace {

// Checks shared by the prepare and GEMM halves.  Returns the first non-empty
// group in *first (-1 when every group is empty).
int check_problem(const FggNvfp4Problem* p, const WsLayout& L, void* workspace, size_t ws_bytes,
                  int* first) {
  if (workspace == nullptr) return set_error(FGG_EINVAL, "workspace is null");
  if (!aligned16(workspace)) return set_error(FGG_EALIGN, "workspace must be 16-byte aligned");
  if (ws_bytes < L.total)
    return set_error(FGG_EWORKSPACE, "workspace has %zu bytes, needs %zu", ws_bytes, L.total);
  if (p->alpha == nullptr || p->a == nullptr || p->a_sf == nullptr)
    return set_error(FGG_EINVAL, "alpha / a / a_sf is null");
  if (L.num_tiles > 0 && p->out == nullptr) return set_error(FGG_EINVAL, "out is null");
  if (p->out != nullptr && !aligned16(p->out))
    return set_error(FGG_EALIGN, "out is not 16-byte aligned");
  *first = -1;
  for (int g = 0; g < p->num_groups; ++g) {
    if (p->m[g] == 0) continue;
    if (p->a[g] == nullptr || p->a_sf[g] == nullptr)
      return set_error(FGG_EINVAL, "group %d activation pointer is null", g);
    if (!aligned16(p->a[g])) return set_error(FGG_EALIGN, "a[%d] is not 16-byte aligned", g);
    if (!aligned4(p->a_sf[g])) return set_error(FGG_EALIGN, "a_sf[%d] is not 4-byte aligned", g);
    if (*first < 0) *first = g;
  }
  return FGG_OK;
}

template <int CAP>
int prepare_launch(const FggNvfp4Problem* p, const WsLayout& L, int first, uint8_t* ws,
                   cudaStream_t s) {
  const int G = p->num_groups;
  static thread_local PrepParams<CAP> pp;  // up to ~17 KB: keep it off the stack
  memset(&pp, 0, sizeof(pp));
  if (int rc = encode_u8_2d(&pp.tmpl, p->a[first], uint64_t(p->k) / 2, uint64_t(p->m[first]), 128,
                            uint32_t(L.box_rows)))
    return rc;
  for (int g = 0; g < G; ++g) {
    pp.a[g] = static_cast<const uint8_t*>(p->a[g]);
    pp.a_sf[g] = static_cast<const uint8_t*>(p->a_sf[g]);
    pp.m[g] = p->m[g];
    pp.out_row[g] = L.out_row[g];
    pp.wgroup[g] = p->b_index != nullptr ? p->b_index[g] : g;
  }
  for (int g = 0; g <= G; ++g) {
    pp.xtile_begin[g] = L.xtile_begin[g];
    pp.tile_begin[g] = L.tile_begin[g];
  }
  pp.tmap_out = reinterpret_cast<CUtensorMap*>(ws + L.tmaps);
  pp.ginfo_out = reinterpret_cast<GroupInfo*>(ws + L.ginfo);
  pp.tiles_out = reinterpret_cast<uint32_t*>(ws + L.tiles);
  pp.sfx_out = ws + L.sfx;
  pp.status = reinterpret_cast<int*>(ws + L.status);
  pp.g = G;
  pp.k = p->k;
  pp.bn = L.bn;
  pp.ch = L.ch;
  pp.nk64p = L.nk64p;
  pp.nt = L.nt;
  pp.num_tiles = L.num_tiles;
  pp.xt_total = L.xt_total;
  pp.blocks_tmap = (G + 7) / 8;
  pp.blocks_tiles = (L.num_tiles + 255) / 256;
  pp.across_groups = L.across_groups ? 1 : 0;
  bool vec = p->k % 256 == 0;
  for (int g = 0; g < G && vec; ++g)
    vec = p->m[g] == 0 || aligned16(p->a_sf[g]);
  pp.sf_vec = vec ? 1 : 0;
  // threads of the scale repack: one per atom row, or per 4 atom rows (vector)
  const int64_t sf_lines = int64_t(L.xt_total) * L.nk64p * L.ch * 32 / (vec ? 4 : 1);
  const int64_t blocks = int64_t(pp.blocks_tmap) + pp.blocks_tiles + (sf_lines + 255) / 256;
  if (blocks > INT32_MAX) return set_error(FGG_EBADSHAPE, "problem too large");
  FGG_CUDA_CHECK(launch_dependent(nvfp4_prepare_kernel<CAP>, int(blocks), 0, s, pp));
  FGG_CUDA_CHECK(cudaGetLastError());
  return FGG_OK;
}

constexpr int kPrepSmallCap = 32;

int prepare_impl(const FggNvfp4Problem* p, const WsLayout& L, int first, uint8_t* ws,
                 cudaStream_t s) {
  if (L.num_tiles == 0) {
    FGG_CUDA_CHECK(cudaMemsetAsync(ws + L.status, 0, kStatusBytes, s));
    return FGG_OK;
  }
  if (p->num_groups <= kPrepSmallCap) return prepare_launch<kPrepSmallCap>(p, L, first, ws, s);
  return prepare_launch<FGG_MAX_GROUPS>(p, L, first, ws, s);
}

int gemm_impl(const FggNvfp4Problem* p, const WsLayout& L, const void* pack, uint8_t* ws,
              const DeviceInfo& dev, cudaStream_t s, int32_t epi = kEpiPlain) {
  if (L.num_tiles == 0) return FGG_OK;
  if (pack == nullptr) return set_error(FGG_EINVAL, "pack is null");
  if (!aligned16(pack)) return set_error(FGG_EALIGN, "pack must be 16-byte aligned");
  const int G = p->num_groups;
  const uint8_t* pk = static_cast<const uint8_t*>(pack);
  const PackLayout PL = pack_layout(L.wg, p->n, p->k);
  GemmParams gp;
  memset(&gp, 0, sizeof(gp));
  gp.tmap_w = reinterpret_cast<const CUtensorMap*>(pk + PL.tmaps);
  gp.tmap_x = reinterpret_cast<const CUtensorMap*>(ws + L.tmaps);
  gp.sfw = pk + PL.sfw;
  gp.sfx = ws + L.sfx;
  gp.ginfo = reinterpret_cast<const GroupInfo*>(ws + L.ginfo);
  gp.tiles = reinterpret_cast<const uint32_t*>(ws + L.tiles);
  gp.alpha = p->alpha;
  gp.pack = reinterpret_cast<const PackHeader*>(pk + PL.header);
  gp.out = static_cast<__nv_bfloat16*>(p->out);
  gp.status = reinterpret_cast<int*>(ws + L.status);
  gp.g = G;
  gp.wg = L.wg;
  gp.n = p->n;
  gp.epi = epi;
  gp.k = p->k;
  gp.m_total = 0;
  gp.num_tiles = L.num_tiles;
  gp.ksteps = L.nk256;
  gp.nt = L.nt;
  gp.nt128 = L.nt128;
  gp.debug_flags = debug_flags();
  cudaError_t e;
  if (L.pair) {
    // scale atoms as rows of uint64: a CTA's 4 weight atoms of a K step are one
    // 2 KB row of the pack, the 8 token atoms of a K step two 2 KB rows
    if (int rc = encode_u64_rows(&gp.sfw_map, gp.sfw,
                                 uint64_t(L.wg) * L.nt128 * L.nk256 * CfgPair::SFW_BOX_ROWS,
                                 CfgPair::SFW_ROW_U64, CfgPair::SFW_BOX_ROWS))
      return rc;
    if (int rc = encode_u64_rows(&gp.sfx_map, gp.sfx,
                                 uint64_t(L.xt_total) * L.nk256 * CfgPair::SFX_BOX_ROWS,
                                 CfgPair::SFX_ROW_U64, CfgPair::SFX_BOX_ROWS))
      return rc;
    e = launch_pair<CfgPair>(gp, dev.sm_count, s);
  } else if (L.bn == CfgDecode::BN) {
    e = launch_engine<CfgDecode>(gp, dev.sm_count, s);
  } else {
    e = launch_engine<CfgPrefill>(gp, dev.sm_count, s);
  }
  if (e != cudaSuccess) return set_error(FGG_ECUDA, "GEMM launch failed: %s", cudaGetErrorString(e));
  return FGG_OK;
}

}  // namespace
}  // namespace fgg

extern "C" {

int fgg_nvfp4_prepare(const FggNvfp4Problem* p, void* workspace, size_t ws_bytes, void* stream) {
  WsLayout L;
  if (int rc = plan(p, &L)) return rc;
  int first = -1;
  if (int rc = check_problem(p, L, workspace, ws_bytes, &first)) return rc;
  DeviceInfo dev;
  if (int rc = current_device(&dev)) return rc;
  return prepare_impl(p, L, first, static_cast<uint8_t*>(workspace),
                      reinterpret_cast<cudaStream_t>(stream));
}

int fgg_nvfp4_gemm(const FggNvfp4Problem* p, const void* pack, void* workspace, size_t ws_bytes,
                   void* stream) {
  WsLayout L;
  if (int rc = plan(p, &L)) return rc;
  int first = -1;
  if (int rc = check_problem(p, L, workspace, ws_bytes, &first)) return rc;
  DeviceInfo dev;
  if (int rc = current_device(&dev)) return rc;
  return gemm_impl(p, L, pack, static_cast<uint8_t*>(workspace), dev,
                   reinterpret_cast<cudaStream_t>(stream));
}

int fgg_nvfp4_grouped_gemm(const FggNvfp4Problem* p, const void* pack, void* workspace,
                           size_t ws_bytes, void* stream) {
  WsLayout L;
  if (int rc = plan(p, &L)) return rc;
  int first = -1;
  if (int rc = check_problem(p, L, workspace, ws_bytes, &first)) return rc;
  if (L.num_tiles > 0 && pack == nullptr) return set_error(FGG_EINVAL, "pack is null");
  DeviceInfo dev;
  if (int rc = current_device(&dev)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (int rc = prepare_impl(p, L, first, ws, s)) return rc;
  return gemm_impl(p, L, pack, ws, dev, s);
}

int fgg_nvfp4_grouped_gemm_silu_mul(const FggNvfp4Problem* p, const void* pack, void* workspace,
                                    size_t ws_bytes, void* stream) {
  WsLayout L;
  if (int rc = plan(p, &L)) return rc;
  if (p->n % 32 != 0)
    return set_error(FGG_EBADSHAPE, "N=%d: gate and up rows come in chunks of 16 + 16", p->n);
  int first = -1;
  if (int rc = check_problem(p, L, workspace, ws_bytes, &first)) return rc;
  if (L.num_tiles > 0 && pack == nullptr) return set_error(FGG_EINVAL, "pack is null");
  DeviceInfo dev;
  if (int rc = current_device(&dev)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (int rc = prepare_impl(p, L, first, ws, s)) return rc;
  return gemm_impl(p, L, pack, ws, dev, s, kEpiSiluMul);
}

}  // extern "C"

namespace fgg {
namespace {

struct RowsLayout {
  int bn = 0, ch = 0, nk64p = 0, nk256 = 0, nt = 0, nt128 = 0, xt_cap = 0, tile_cap = 0;
  bool pair = false, decode = false;
  int box_rows = 0;
  size_t status = 0, ginfo = 0, tiles = 0, sfx = 0, total = 0;
};

int plan_rows(const FggNvfp4RowsProblem* p, RowsLayout* L) {
  if (p == nullptr) return set_error(FGG_EINVAL, "problem is null");
  const int G = p->num_groups;
  if (G < 1 || G > FGG_MAX_GROUPS)
    return set_error(FGG_EINVAL, "num_groups=%d outside [1, %d]", G, FGG_MAX_GROUPS);
  if (p->n <= 0 || p->n % 128 != 0)
    return set_error(FGG_EBADSHAPE, "N=%d must be a positive multiple of 128", p->n);
  if (p->k < 64 || p->k % 64 != 0)
    return set_error(FGG_EBADSHAPE, "K=%d must be a positive multiple of 64", p->k);
  if (p->n / 128 > 2047) return set_error(FGG_EBADSHAPE, "N=%d too large", p->n);
  if (p->max_rows < 0) return set_error(FGG_EINVAL, "max_rows=%d is negative", p->max_rows);
  if (p->b_index != nullptr &&
      (p->num_weight_groups < 1 || p->num_weight_groups > FGG_MAX_GROUPS))
    return set_error(FGG_EINVAL, "num_weight_groups=%d outside [1, %d]", p->num_weight_groups,
                     FGG_MAX_GROUPS);
  const int maxg = p->max_group_rows > 0 ? std::min(p->max_group_rows, p->max_rows) : p->max_rows;
  L->decode = maxg <= 16;
  L->pair = !L->decode && (p->n % 256 == 0);
  L->bn = L->decode ? CfgDecode::BN : CfgPrefill::BN;
  L->ch = L->decode ? CfgDecode::CH : CfgPrefill::CH;
  L->box_rows = L->pair ? CfgPair::BNH : L->bn;
  L->nk256 = (p->k + 255) / 256;
  L->nk64p = 4 * L->nk256;
  L->nt128 = p->n / 128;
  L->nt = L->pair ? p->n / 256 : L->nt128;
  // token tiles: sum_g ceil(M_g / BN) <= max_rows / BN + G
  const int64_t xt_cap = (int64_t(p->max_rows) + L->bn - 1) / L->bn + G;
  const int64_t tile_cap = xt_cap * L->nt;
  if (xt_cap > INT32_MAX / 2 || tile_cap > INT32_MAX) return set_error(FGG_EBADSHAPE, "problem too large");
  if (int64_t(maxg + L->bn - 1) / L->bn > 2047)
    return set_error(FGG_EBADSHAPE, "groups of up to %d rows are too large", maxg);
  L->xt_cap = int(xt_cap);
  L->tile_cap = int(tile_cap);
  Carver cv;
  L->status = cv.take(kStatusBytes, 256);
  L->ginfo = cv.take(size_t(G) * sizeof(GroupInfo), 256);
  L->tiles = cv.take(size_t(std::max<int64_t>(tile_cap, 1)) * 4, 256);
  L->sfx = cv.take(size_t(std::max<int64_t>(xt_cap, 1)) * L->nk64p * L->ch * 512, 256);
  L->total = cv.off;
  return FGG_OK;
}

}  // namespace
}  // namespace fgg

extern "C" {

size_t fgg_nvfp4_rows_workspace_bytes(const FggNvfp4RowsProblem* p) {
  RowsLayout L;
  if (plan_rows(p, &L) != FGG_OK) return 0;
  return L.total;
}

int fgg_nvfp4_grouped_gemm_rows(const FggNvfp4RowsProblem* p, const void* pack, void* workspace,
                                size_t ws_bytes, void* stream) {
  RowsLayout L;
  if (int rc = plan_rows(p, &L)) return rc;
  if (workspace == nullptr) return set_error(FGG_EINVAL, "workspace is null");
  if (!aligned16(workspace)) return set_error(FGG_EALIGN, "workspace must be 16-byte aligned");
  if (ws_bytes < L.total)
    return set_error(FGG_EWORKSPACE, "workspace has %zu bytes, needs %zu", ws_bytes, L.total);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (p->max_rows == 0) {
    FGG_CUDA_CHECK(cudaMemsetAsync(ws + L.status, 0, kStatusBytes, s));
    return FGG_OK;
  }
  if (p->offsets == nullptr || p->a == nullptr || p->a_sf == nullptr || p->alpha == nullptr ||
      p->out == nullptr)
    return set_error(FGG_EINVAL, "offsets / a / a_sf / alpha / out is null");
  if (pack == nullptr) return set_error(FGG_EINVAL, "pack is null");
  if (!aligned16(p->a) || !aligned16(p->out) || !aligned16(pack))
    return set_error(FGG_EALIGN, "a, out and pack must be 16-byte aligned");
  if (!aligned4(p->a_sf) || !aligned4(p->offsets) || !aligned4(p->alpha) ||
      (p->row_scale != nullptr && !aligned4(p->row_scale)) ||
      (p->b_index != nullptr && !aligned4(p->b_index)))
    return set_error(FGG_EALIGN, "a_sf, offsets, alpha, row_scale and b_index must be 4-byte aligned");
  DeviceInfo dev;
  if (int rc = current_device(&dev)) return rc;
  const int G = p->num_groups;
  const int wg = p->b_index != nullptr ? p->num_weight_groups : G;

  RowsPrepParams pp;
  memset(&pp, 0, sizeof(pp));
  pp.offsets = p->offsets;
  pp.b_index = p->b_index;
  pp.a_sf = static_cast<const uint8_t*>(p->a_sf);
  pp.ginfo_out = reinterpret_cast<GroupInfo*>(ws + L.ginfo);
  pp.tiles_out = reinterpret_cast<uint32_t*>(ws + L.tiles);
  pp.sfx_out = ws + L.sfx;
  pp.status = reinterpret_cast<int*>(ws + L.status);
  pp.g = G;
  pp.wg = wg;
  pp.k = p->k;
  pp.bn = L.bn;
  pp.ch = L.ch;
  pp.nk64p = L.nk64p;
  pp.nt = L.nt;
  pp.max_rows = p->max_rows;
  pp.tile_cap = L.tile_cap;
  pp.xt_cap = L.xt_cap;
  pp.blocks_tiles = (L.tile_cap + 255) / 256;
  pp.sf_vec = (p->k % 256 == 0 && aligned16(p->a_sf)) ? 1 : 0;
  pp.decode = L.decode ? 1 : 0;
  const int64_t sf_lines = int64_t(L.xt_cap) * L.nk64p * L.ch * 32 / (pp.sf_vec ? 4 : 1);
  const int64_t blocks = 1 + int64_t(pp.blocks_tiles) + (sf_lines + 255) / 256;
  if (blocks > INT32_MAX) return set_error(FGG_EBADSHAPE, "problem too large");
  FGG_CUDA_CHECK(launch_dependent(nvfp4_prepare_rows_kernel, int(blocks), 0, s, pp));
  FGG_CUDA_CHECK(cudaGetLastError());

  const uint8_t* pk = static_cast<const uint8_t*>(pack);
  const PackLayout PL = pack_layout(wg, p->n, p->k);
  GemmParams gp;
  memset(&gp, 0, sizeof(gp));
  if (int rc = encode_u8_2d(&gp.tmap_x_flat, p->a, uint64_t(p->k) / 2, uint64_t(p->max_rows), 128,
                            uint32_t(L.box_rows)))
    return rc;
  gp.x_flat = 1;
  gp.tmap_w = reinterpret_cast<const CUtensorMap*>(pk + PL.tmaps);
  gp.sfw = pk + PL.sfw;
  gp.sfx = ws + L.sfx;
  gp.ginfo = reinterpret_cast<const GroupInfo*>(ws + L.ginfo);
  gp.tiles = reinterpret_cast<const uint32_t*>(ws + L.tiles);
  gp.alpha = p->alpha;
  gp.row_scale = p->row_scale;
  gp.pack = reinterpret_cast<const PackHeader*>(pk + PL.header);
  gp.out = static_cast<__nv_bfloat16*>(p->out);
  gp.status = reinterpret_cast<int*>(ws + L.status);
  gp.num_tiles_dev = reinterpret_cast<const int32_t*>(ws + L.status) + 3;
  gp.g = G;
  gp.wg = wg;
  gp.n = p->n;
  gp.k = p->k;
  gp.epi = kEpiPlain;
  gp.num_tiles = L.tile_cap;  // the launch's grid bound; the kernels read the real count
  gp.ksteps = L.nk256;
  gp.nt = L.nt;
  gp.nt128 = L.nt128;
  gp.debug_flags = debug_flags();
  cudaError_t e;
  if (L.pair) {
    if (int rc = encode_u64_rows(&gp.sfw_map, gp.sfw,
                                 uint64_t(wg) * L.nt128 * L.nk256 * CfgPair::SFW_BOX_ROWS,
                                 CfgPair::SFW_ROW_U64, CfgPair::SFW_BOX_ROWS))
      return rc;
    if (int rc = encode_u64_rows(&gp.sfx_map, gp.sfx,
                                 uint64_t(L.xt_cap) * L.nk256 * CfgPair::SFX_BOX_ROWS,
                                 CfgPair::SFX_ROW_U64, CfgPair::SFX_BOX_ROWS))
      return rc;
    // the narrow token boxes (a tail tile of a group loads only its rows)
    for (int i = 0; i < kXSmallMaps; ++i)
      if (int rc = encode_u8_2d(&gp.tmap_x_small[i], p->a, uint64_t(p->k) / 2,
                                uint64_t(p->max_rows), 128, uint32_t(16 * (i + 1))))
        return rc;
    gp.x_small = 1;
    e = launch_pair<CfgPair>(gp, dev.sm_count, s);
  } else if (L.decode) {
    e = launch_engine<CfgDecode>(gp, dev.sm_count, s);
  } else {
    e = launch_engine<CfgPrefill>(gp, dev.sm_count, s);
  }
  if (e != cudaSuccess) return set_error(FGG_ECUDA, "GEMM launch failed: %s", cudaGetErrorString(e));
  return FGG_OK;
}

}  // extern "C"

namespace fgg {
int noalloc_scratch(void** out);  // fgg_scratch.cu
}  // namespace fgg

extern "C" {

int fgg_nvfp4_grouped_gemm_noalloc(const FggNvfp4Problem* p, const void* pack, void* status_out,
                                   void* stream) {
  WsLayout L;
  if (int rc = plan(p, &L)) return rc;
  // refused before any device work
  if (L.total > size_t(FGG_NOALLOC_SCRATCH_BYTES))
    return set_error(FGG_EWORKSPACE,
                     "problem needs %zu bytes of scratch, the static scratch holds %zu; "
                     "use fgg_nvfp4_grouped_gemm with a caller workspace",
                     L.total, size_t(FGG_NOALLOC_SCRATCH_BYTES));
  if (status_out != nullptr && !aligned4(status_out))
    return set_error(FGG_EALIGN, "status_out is not 4-byte aligned");
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  int first = -1;
  if (int rc = check_problem(p, L, scratch, size_t(FGG_NOALLOC_SCRATCH_BYTES), &first)) return rc;
  if (L.num_tiles > 0 && pack == nullptr) return set_error(FGG_EINVAL, "pack is null");
  DeviceInfo dev;
  if (int rc = current_device(&dev)) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(scratch);
  if (int rc = prepare_impl(p, L, first, ws, s)) return rc;
  if (int rc = gemm_impl(p, L, pack, ws, dev, s)) return rc;
  if (status_out != nullptr)
    FGG_CUDA_CHECK(
        cudaMemcpyAsync(status_out, ws + L.status, sizeof(int32_t), cudaMemcpyDeviceToDevice, s));
  return FGG_OK;
}

}  // extern "C"
