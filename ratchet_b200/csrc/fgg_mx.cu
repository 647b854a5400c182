// fgg_mx.cu - MXFP8 x MXFP4 contiguous M-grouped GEMM, the reference operator
// `fp4_grouped_gemm(a, a_sf, b, b_sf, m_indices)`
// (kernels/gemm/fp4_grouped_gemm/b200/kernel.py:2788-2862), on the shared
// tcgen05 engine with .kind::mxf8f6f4.
//
// Per call (unless the caller marks the workspace as already prepared):
//   mx_prepare_kernel
//     - block -> expert table from m_indices[224 * i] (kernel.py:2780), fused
//       straight into the flat tile list
//     - activation scales (fp32 powers of two, one per 1x128) -> UE8M0 bytes,
//       each replicated into the four K32 slots of the SF atom
//       (kernel.py:2679-2707)
//     - weight scales (one per 1x32) -> UE8M0 SF atoms (kernel.py:2709-2741)
//   fgg_gemm_kernel<MX cfg>
#include <algorithm>
#include <cstring>

#include "fgg_engine.cuh"
#include "fgg_host.cuh"

namespace fgg {

namespace {

constexpr int kMxBlockM = 224;  // token tile = the reference's ALIGN (kernel.py:274)

using CfgMx = EngineCfg<true, kMxBlockM, 4>;  // one CTA per tile (N % 256 != 0)
using CfgMxPair = PairCfg<true, 7>;          // CTA pairs, 256 x 224 tiles

struct MxPrepParams {
  const float* a_sf;        // [M_total, K/128]
  const float* b_sf;        // [G, N, K/32]
  const int32_t* m_indices; // [M_total]
  uint8_t* sfx_out;         // [XB][KS][2][512]
  uint8_t* sfw_out;         // [G][NT][KS][512]
  uint32_t* tiles_out;      // [XB * NT]
  int* status;
  int32_t m_total, n, k, g, nt, nt128, ksteps, xblocks;
  int32_t blocks_tiles, blocks_sfx;
};

// UE8M0 byte of an fp32 power of two: its exponent field (kernel.py:2679-2681).
__device__ __forceinline__ uint32_t e8m0_byte(float v) {
  return (__float_as_uint(v) >> 23) & 0xFFu;
}

__global__ void __launch_bounds__(256) mx_prepare_kernel(const __grid_constant__ MxPrepParams p) {
  // every block is resident once it gets here: the GEMM grid behind this one
  // may launch now (it waits for this grid's results before reading them)
  griddep_launch_dependents();
  // launched early behind the previous GEMM: touch no memory before it is done
  griddep_wait();
  int blk = blockIdx.x;
  if (blk < p.blocks_tiles) {
    if (blk == 0 && threadIdx.x == 0) {
      p.status[0] = 0;
      p.status[1] = 0;
      p.status[2] = 0;
    }
    const int t = blk * blockDim.x + threadIdx.x;
    if (t < p.xblocks * p.nt) {
      const int xb = t / p.nt;
      const int nti = t - xb * p.nt;
      int e = __ldg(p.m_indices + size_t(xb) * kMxBlockM);
      e = min(max(e, 0), p.g - 1);  // padding block -> expert 0 (output unchecked)
      p.tiles_out[t] = pack_tile(e, nti, xb);
    }
    return;
  }
  blk -= p.blocks_tiles;
  const int kq = p.k / 128;  // activation scales per row
  if (blk < p.blocks_sfx) {
    // one 16-byte atom row: rows c*128 + r1*32 + r0 (r1 = 0..3) of block xb
    const int64_t line = int64_t(blk) * blockDim.x + threadIdx.x;
    if (line >= int64_t(p.xblocks) * p.ksteps * 2 * 32) return;
    const int r0 = int(line & 31);
    int64_t rest = line >> 5;
    const int c = int(rest & 1);
    rest >>= 1;
    const int ks = int(rest % p.ksteps);
    const int xb = int(rest / p.ksteps);
    uint32_t v[4];
#pragma unroll
    for (int r1 = 0; r1 < 4; ++r1) {
      const int rr = c * 128 + r1 * 32 + r0;
      const int row = xb * kMxBlockM + rr;
      v[r1] = 0u;
      if (rr < kMxBlockM && row < p.m_total)
        v[r1] = e8m0_byte(__ldg(p.a_sf + size_t(row) * kq + ks)) * 0x01010101u;
    }
    *reinterpret_cast<uint4*>(p.sfx_out + ((size_t(xb) * p.ksteps + ks) * 2 + c) * 512u +
                              size_t(r0) * 16u) = make_uint4(v[0], v[1], v[2], v[3]);
    return;
  }
  blk -= p.blocks_sfx;
  {
    const int64_t line = int64_t(blk) * blockDim.x + threadIdx.x;
    if (line >= int64_t(p.g) * p.nt128 * p.ksteps * 32) return;
    const int r0 = int(line & 31);
    int64_t rest = line >> 5;
    const int ks = int(rest % p.ksteps);
    rest /= p.ksteps;
    const int nti = int(rest % p.nt128);
    const int g = int(rest / p.nt128);
    const int kw = p.k / 32;  // weight scales per row
    uint32_t v[4];
#pragma unroll
    for (int r1 = 0; r1 < 4; ++r1) {
      const int row = nti * 128 + r1 * 32 + r0;
      const float4 s = __ldg(reinterpret_cast<const float4*>(p.b_sf + (size_t(g) * p.n + row) * kw +
                                                             size_t(ks) * 4));
      v[r1] = e8m0_byte(s.x) | (e8m0_byte(s.y) << 8) | (e8m0_byte(s.z) << 16) |
              (e8m0_byte(s.w) << 24);
    }
    uint4* dst = reinterpret_cast<uint4*>(
        p.sfw_out + ((size_t(g) * p.nt128 + nti) * p.ksteps + ks) * 512u + size_t(r0) * 16u);
    *dst = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

struct MxLayout {
  bool pair = false;
  int xblocks = 0, nt = 0, nt128 = 0, ksteps = 0, num_tiles = 0;
  size_t status = 0, tiles = 0, sfx = 0, sfw = 0, total = 0;
};

int mx_plan(const FggMxProblem* p, MxLayout* L) {
  if (p == nullptr) return set_error(FGG_EINVAL, "problem is null");
  if (p->num_groups < 1 || p->num_groups > 1023)
    return set_error(FGG_EINVAL, "num_groups=%d outside [1, 1023]", p->num_groups);
  if (p->m_total < 0) return set_error(FGG_EINVAL, "m_total=%d is negative", p->m_total);
  // kernel.py:2811-2816
  if (p->n <= 0 || p->n % 128 != 0)
    return set_error(FGG_EBADSHAPE, "N=%d is not a multiple of BLOCK_N=128", p->n);
  if (p->k <= 0 || p->k % 128 != 0)
    return set_error(FGG_EBADSHAPE, "K=%d is not a multiple of BLOCK_K=128", p->k);
  L->xblocks = (p->m_total + kMxBlockM - 1) / kMxBlockM;
  L->pair = (p->n % 256 == 0);
  L->nt128 = p->n / 128;
  L->nt = L->pair ? p->n / 256 : L->nt128;
  L->ksteps = p->k / 128;
  if (L->xblocks > 2047 || L->nt > 2047) return set_error(FGG_EBADSHAPE, "problem too large");
  L->num_tiles = L->xblocks * L->nt;
  Carver cv;
  L->status = cv.take(kStatusBytes, 256);
  L->tiles = cv.take(size_t(std::max(L->num_tiles, 1)) * 4, 256);
  L->sfx = cv.take(size_t(std::max(L->xblocks, 1)) * L->ksteps * 1024, 256);
  L->sfw = cv.take(size_t(p->num_groups) * L->nt128 * L->ksteps * 512, 256);
  L->total = cv.off;
  return FGG_OK;
}

}  // namespace
}  // namespace fgg

using namespace fgg;

extern "C" {

size_t fgg_mx_workspace_bytes(const FggMxProblem* p) {
  MxLayout L;
  if (mx_plan(p, &L) != FGG_OK) return 0;
  return L.total;
}

int fgg_mx_grouped_gemm(const FggMxProblem* p, void* workspace, size_t ws_bytes, void* stream) {
  MxLayout L;
  if (int rc = mx_plan(p, &L)) return rc;
  if (workspace == nullptr) return set_error(FGG_EINVAL, "workspace is null");
  if (!aligned16(workspace)) return set_error(FGG_EALIGN, "workspace is not 16-byte aligned");
  if (ws_bytes < L.total)
    return set_error(FGG_EWORKSPACE, "workspace has %zu bytes, needs %zu", ws_bytes, L.total);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (L.num_tiles == 0) {
    FGG_CUDA_CHECK(cudaMemsetAsync(ws + L.status, 0, kStatusBytes, s));
    return FGG_OK;
  }
  if (p->a == nullptr || p->a_sf == nullptr || p->b == nullptr || p->b_sf == nullptr ||
      p->m_indices == nullptr || p->c == nullptr)
    return set_error(FGG_EINVAL, "a null operand pointer");
  if (!aligned16(p->a) || !aligned16(p->c) || !aligned16(p->b_sf) || !aligned4(p->a_sf) ||
      !aligned4(p->m_indices))
    return set_error(FGG_EALIGN, "operands must be 16-byte aligned (a_sf, m_indices: 4-byte)");
  if ((reinterpret_cast<uintptr_t>(p->b) & 31u) != 0)
    return set_error(FGG_EALIGN, "b must be 32-byte aligned (4-bit TMA unpack)");
  DeviceInfo dev;
  if (int rc = current_device(&dev)) return rc;

  if (!p->reuse_prepared) {
    MxPrepParams pp;
    memset(&pp, 0, sizeof(pp));
    pp.a_sf = p->a_sf;
    pp.b_sf = p->b_sf;
    pp.m_indices = p->m_indices;
    pp.sfx_out = ws + L.sfx;
    pp.sfw_out = ws + L.sfw;
    pp.tiles_out = reinterpret_cast<uint32_t*>(ws + L.tiles);
    pp.status = reinterpret_cast<int*>(ws + L.status);
    pp.m_total = p->m_total;
    pp.n = p->n;
    pp.k = p->k;
    pp.g = p->num_groups;
    pp.nt = L.nt;
    pp.nt128 = L.nt128;
    pp.ksteps = L.ksteps;
    pp.xblocks = L.xblocks;
    pp.blocks_tiles = (L.num_tiles + 255) / 256;
    pp.blocks_sfx = int((int64_t(L.xblocks) * L.ksteps * 64 + 255) / 256);
    const int64_t sfw_lines = int64_t(p->num_groups) * L.nt128 * L.ksteps * 32;
    const int64_t blocks = int64_t(pp.blocks_tiles) + pp.blocks_sfx + (sfw_lines + 255) / 256;
    FGG_CUDA_CHECK(launch_dependent(mx_prepare_kernel, int(blocks), 0, s, pp));
    FGG_CUDA_CHECK(cudaGetLastError());
  } else {
    // the prepare kernel, skipped here, is what clears the status words: a
    // reused workspace must not carry an earlier call's status into this one
    FGG_CUDA_CHECK(cudaMemsetAsync(ws + L.status, 0, 3 * sizeof(int32_t), s));
  }

  GemmParams gp;
  memset(&gp, 0, sizeof(gp));
  // weights: [G, N, K] 4-bit codes; the 16U4_ALIGN16B type lands each 16 codes
  // (8 bytes) in a 16-byte slot, the byte-container form .kind::mxf8f6f4 reads.
  if (int rc = encode_3d(&gp.mx_tmap_w, CU_TENSOR_MAP_DATA_TYPE_16U4_ALIGN16B, p->b,
                         uint64_t(p->k), uint64_t(p->n), uint64_t(p->num_groups),
                         uint64_t(p->k) / 2, uint64_t(p->n) * uint64_t(p->k) / 2, 128, 128, 1))
    return rc;
  if (int rc = encode_2d(&gp.tmap_x_flat, CU_TENSOR_MAP_DATA_TYPE_UINT8, p->a, uint64_t(p->k),
                         uint64_t(p->m_total), uint64_t(p->k), 128,
                         L.pair ? CfgMxPair::BNH : kMxBlockM))
    return rc;
  gp.sfw = ws + L.sfw;
  gp.sfx = ws + L.sfx;
  gp.tiles = reinterpret_cast<const uint32_t*>(ws + L.tiles);
  gp.out = static_cast<__nv_bfloat16*>(p->c);
  gp.status = reinterpret_cast<int*>(ws + L.status);
  gp.g = p->num_groups;
  gp.wg = p->num_groups;
  gp.n = p->n;
  gp.k = p->k;
  gp.m_total = p->m_total;
  gp.num_tiles = L.num_tiles;
  gp.ksteps = L.ksteps;
  gp.nt = L.nt;
  gp.nt128 = L.nt128;
  gp.debug_flags = debug_flags();
  cudaError_t e;
  if (L.pair) {
    if (int rc = encode_u64_rows(&gp.sfw_map, gp.sfw,
                                 uint64_t(p->num_groups) * L.nt128 * L.ksteps,
                                 CfgMxPair::SFW_ROW_U64, CfgMxPair::SFW_BOX_ROWS))
      return rc;
    if (int rc = encode_u64_rows(&gp.sfx_map, gp.sfx,
                                 uint64_t(L.xblocks) * L.ksteps * CfgMxPair::SFX_BOX_ROWS,
                                 CfgMxPair::SFX_ROW_U64, CfgMxPair::SFX_BOX_ROWS))
      return rc;
    e = launch_pair<CfgMxPair>(gp, dev.sm_count, s);
  } else {
    e = launch_engine<CfgMx>(gp, dev.sm_count, s);
  }
  if (e != cudaSuccess) return set_error(FGG_ECUDA, "MX GEMM launch failed: %s", cudaGetErrorString(e));
  return FGG_OK;
}

}  // extern "C"
