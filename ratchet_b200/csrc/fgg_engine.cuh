// fgg_engine.cuh - the persistent tcgen05 grouped-GEMM engine shared by both
// operand formats.
//
// Orientation ("swap AB", as kernels/gemm/fp4_grouped_gemm/b200/kernel.py:84-86
// does with MMA-A = weights): the tensor core's M axis runs over 128 weight rows
// (output columns n), its N axis over up to BN tokens of one group (output rows
// m).  Ragged group sizes land on the MMA's N axis, sized per tile in steps of
// 16, and the epilogue's lanes walk consecutive output columns.
//
// One CTA per SM, 256 threads, warp-specialised:
//   warp 0     claims tiles from a global atomic counter (dynamic persistent
//              schedule), broadcasts them through an smem ring, and issues the
//              TMA / bulk loads of every K step into a STAGES-deep ring
//   warp 1     one thread issues tcgen05.cp (scale factors -> TMEM) and the
//              block-scaled tcgen05.mma chain into a double-buffered TMEM
//              accumulator
//   warp 2     allocates / frees TMEM
//   warps 4-7  epilogue: tcgen05.ld (each warp its 32-lane quadrant) -> fp32
//              x alpha -> bf16 -> global, overlapped with the next tile's MMAs
//
// Two kinds (compile-time):
//   NVFP4   .kind::mxf4nvf4 .scale_vec::4X: E2M1 x E2M1, one E4M3 scale per 16
//           K; K step 256 = 4 MMAs of K 64, one SF slot per MMA.
//   MX      .kind::mxf8f6f4: weights E2M1 (4-bit codes unpacked to bytes by
//           TMA), tokens E4M3, one UE8M0 scale per 32 K; K step 128 = 4 MMAs of
//           K 32 that share one SF slot and pick their byte with the SF id.
#pragma once

#include <cuda_bf16.h>

#include "fgg_ptx.cuh"

namespace fgg {

struct GroupInfo {
  int32_t m;            // rows of A_g
  int32_t out_row;      // first output row of the group
  int32_t xtile_begin;  // index of the group's first token tile in the SF repack
  int32_t xtiles;       // token tiles of the group
};

// A tile is packed into 32 bits: group (10) | weight tile (11) | token tile (11).
__host__ __device__ __forceinline__ uint32_t pack_tile(int g, int nt, int xt) {
  return (uint32_t(g) << 22) | (uint32_t(nt) << 11) | uint32_t(xt);
}
constexpr uint32_t kEndTile = 0xFFFFFFFFu;

constexpr uint32_t kPackMagic = 0x46474e34u;  // "FGN4"
struct PackHeader {
  uint32_t magic;
  int32_t g, n, k;
};

constexpr int kStatusBadPack = 0x201;

template <bool MX_, int BN_, int STAGES_>
struct EngineCfg {
  static constexpr bool MX = MX_;
  static constexpr int BN = BN_;
  static constexpr int STAGES = STAGES_;
  static constexpr int CH = (BN + 127) / 128;  // 128-row SF atoms per token tile
  // K elements per pipeline stage: one 128-byte swizzle row of each operand.
  static constexpr int K_STEP = MX ? 128 : 256;
  static constexpr uint32_t W_BYTES = 128 * 128;   // smem bytes of the weight tile
  static constexpr uint32_t W_TX = MX ? 64 * 128 : 128 * 128;  // bytes TMA reads from HBM
  static constexpr uint32_t X_BYTES = BN * 128;
  // NVFP4: 4 atoms (one per K64 MMA); MX: one atom covers the 4 K32 MMAs.
  static constexpr uint32_t SFW_BYTES = MX ? 512 : 4 * 512;
  static constexpr uint32_t SFX_BYTES = MX ? CH * 512 : 4 * CH * 512;
  static constexpr uint32_t TX_BYTES = W_TX + X_BYTES + SFW_BYTES + SFX_BYTES;
  static constexpr uint32_t STAGE_BYTES =
      (W_BYTES + X_BYTES + SFW_BYTES + SFX_BYTES + 1023) / 1024 * 1024;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "BN must be a multiple of 16");
  static_assert((W_BYTES + X_BYTES) % 1024 == 0, "operand tiles must stay 1024 B aligned");
  // TMEM columns: two accumulators of BN fp32 columns, then a ring of scale
  // slots (4 columns of weight scales + 4 per token atom).  NVFP4 takes one
  // slot per MMA, MX one per K step.
  static constexpr int SF_BASE = ((2 * BN + 3) / 4) * 4;
  static constexpr int SF_SLOT = 4 + 4 * CH;
  static constexpr int NSLOTS_FIT = (512 - SF_BASE) / SF_SLOT;
  static constexpr int NSLOTS = NSLOTS_FIT > 8 ? 8 : NSLOTS_FIT;
  static_assert(NSLOTS >= 2, "not enough TMEM for the scale ring");
  static constexpr int COLS = SF_BASE + NSLOTS * SF_SLOT;
  static constexpr uint32_t TMEM_COLS =
      COLS <= 32 ? 32 : COLS <= 64 ? 64 : COLS <= 128 ? 128 : COLS <= 256 ? 256 : 512;
  static constexpr int SCHED = 8;  // tile-broadcast ring depth
  // barriers: full[S] empty[S] accf[2] acce[2] schedf[SCHED] schede[SCHED] tmem_ready drain
  static constexpr uint32_t NBARS = 2 * STAGES + 4 + 2 * SCHED + 2;
  static constexpr uint32_t MISC_BYTES = 8 * NBARS + 4 * SCHED + 16;
  static constexpr uint32_t SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + MISC_BYTES;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

struct GemmParams {
  CUtensorMap mx_tmap_w;      // MX: 3-D map of the [G, N, K] weight codes
  CUtensorMap mx_tmap_x;      // MX: 2-D map of the [M_total, K] fp8 activations
  const CUtensorMap* tmap_w;  // NVFP4: [G] per-group maps (global memory)
  const CUtensorMap* tmap_x;  // NVFP4: [G] per-group maps (global memory)
  const uint8_t* sfw;         // [G][NT][KSTEPS][SFW_BYTES]
  const uint8_t* sfx;         // [XT][KSTEPS][SFX_BYTES]
  const GroupInfo* ginfo;     // NVFP4: [G]
  const uint32_t* tiles;      // [T]
  const float* alpha;         // NVFP4: [G]; MX: unused (1)
  const PackHeader* pack;     // NVFP4: weight pack header; MX: null
  __nv_bfloat16* out;
  int* status;  // [0] status, [1] tile counter, [2] finished CTAs
  int32_t g, n, k;
  int32_t m_total;  // MX: rows of the contiguous activation tensor
  int32_t num_tiles;
  int32_t ksteps;
  int32_t nt;
};

template <class C>
__global__ void __launch_bounds__(256, 1) fgg_gemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);

  const uint32_t bars = base + C::STAGES * C::STAGE_BYTES;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (C::STAGES + s); };
  auto accf_bar = [&](int b) { return bars + 8u * (2 * C::STAGES + b); };
  auto acce_bar = [&](int b) { return bars + 8u * (2 * C::STAGES + 2 + b); };
  auto schedf_bar = [&](int i) { return bars + 8u * (2 * C::STAGES + 4 + i); };
  auto schede_bar = [&](int i) { return bars + 8u * (2 * C::STAGES + 4 + C::SCHED + i); };
  const uint32_t tmem_ready_bar = bars + 8u * (2 * C::STAGES + 4 + 2 * C::SCHED);
  const uint32_t drain_bar = tmem_ready_bar + 8u;
  uint8_t* const misc = gbase + C::STAGES * C::STAGE_BYTES + 8 * C::NBARS;
  volatile uint32_t* const sched_tile = reinterpret_cast<volatile uint32_t*>(misc);
  volatile uint32_t* const tmem_holder = reinterpret_cast<volatile uint32_t*>(misc + 4 * C::SCHED);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(misc + 4 * C::SCHED + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  auto sW = [&](int s) { return base + s * C::STAGE_BYTES; };
  auto sX = [&](int s) { return base + s * C::STAGE_BYTES + C::W_BYTES; };
  auto sSFW = [&](int s) { return base + s * C::STAGE_BYTES + C::W_BYTES + C::X_BYTES; };
  auto sSFX = [&](int s) {
    return base + s * C::STAGE_BYTES + C::W_BYTES + C::X_BYTES + C::SFW_BYTES;
  };

  // rows of the token tile and the bf16 output base of its first row
  auto tile_rows = [&](int g, int xti) -> int {
    if constexpr (C::MX) {
      return min(C::BN, p.m_total - xti * C::BN);
    } else {
      return min(C::BN, p.ginfo[g].m - xti * C::BN);
    }
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), 4);  // one arrival per epilogue warp
    }
    for (int i = 0; i < C::SCHED; ++i) {
      mbar_init(schedf_bar(i), 1);
      mbar_init(schede_bar(i), 5);  // MMA warp + 4 epilogue warps
    }
    mbar_init(tmem_ready_bar, 1);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    if constexpr (!C::MX) {
      // A pack built for a different problem is refused before any load.
      const PackHeader h = *p.pack;
      if (h.magic != kPackMagic || h.g != p.g || h.n != p.n || h.k != p.k) {
        atomicCAS(p.status, 0, kStatusBadPack);
        *abort_flag = 1;
      }
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 2) {
    tmem_alloc(smem_u32(const_cast<uint32_t*>(tmem_holder)), C::TMEM_COLS);
    tmem_relinquish();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(tmem_ready_bar);
  }

  const bool aborted_early = (*abort_flag != 0);

  if (warp == 0 && !aborted_early) {
    // ------------------------------------------------ producer + scheduler
    int stage = 0;
    uint32_t phase = 0;
    int slot = 0;
    uint32_t sphase = 0;
    uint32_t arms = 0;
    if constexpr (C::MX) {
      if (lane == 0) {
        prefetch_tensormap(&p.mx_tmap_w);
        prefetch_tensormap(&p.mx_tmap_x);
      }
    }
    while (true) {
      int t = 0;
      if (lane == 0) t = atomicAdd(p.status + 1, 1);
      t = __shfl_sync(0xffffffffu, t, 0);
      const uint32_t tile = (t < p.num_tiles) ? p.tiles[t] : kEndTile;
      if (!mbar_wait(schede_bar(slot), sphase ^ 1, abort_flag, p.status, kStatusTimeoutProducer))
        break;
      if (lane == 0) {
        sched_tile[slot] = tile;
        mbar_arrive(schedf_bar(slot));
      }
      __syncwarp();
      if (++slot == C::SCHED) {
        slot = 0;
        sphase ^= 1;
      }
      if (tile == kEndTile) break;
      const int g = int(tile >> 22);
      const int nti = int((tile >> 11) & 0x7FFu);
      const int xti = int(tile & 0x7FFu);
      const CUtensorMap* tw;
      const CUtensorMap* tx;
      const uint8_t* sfx;
      if constexpr (C::MX) {
        tw = &p.mx_tmap_w;
        tx = &p.mx_tmap_x;
        sfx = p.sfx + size_t(xti) * size_t(p.ksteps) * C::SFX_BYTES;
      } else {
        tw = p.tmap_w + g;
        tx = p.tmap_x + g;
        sfx = p.sfx + size_t(p.ginfo[g].xtile_begin + xti) * size_t(p.ksteps) * C::SFX_BYTES;
        if (lane == 0) {
          tensormap_acquire(tw);
          tensormap_acquire(tx);
        }
      }
      const uint8_t* sfw = p.sfw + (size_t(g) * p.nt + nti) * size_t(p.ksteps) * C::SFW_BYTES;
      bool ok = true;
      for (int ks = 0; ks < p.ksteps; ++ks) {
        if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.status,
                       kStatusTimeoutProducer)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, C::TX_BYTES);
          if constexpr (C::MX) {
            tma_load_3d(sW(stage), tw, fb, ks * C::K_STEP, nti * 128, g);
            tma_load_2d(sX(stage), tx, fb, ks * C::K_STEP, xti * C::BN);
          } else {
            tma_load_2d(sW(stage), tw, fb, ks * 128, nti * 128);
            tma_load_2d(sX(stage), tx, fb, ks * 128, xti * C::BN);
          }
          bulk_g2s(sSFW(stage), sfw + size_t(ks) * C::SFW_BYTES, C::SFW_BYTES, fb);
          bulk_g2s(sSFX(stage), sfx + size_t(ks) * C::SFX_BYTES, C::SFX_BYTES, fb);
        }
        __syncwarp();
        ++arms;
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
    }
    // Every armed stage must land before the CTA may exit (normally already so).
    if (lane == 0) {
      const uint32_t first = arms > uint32_t(C::STAGES) ? arms - C::STAGES : 0u;
      for (uint32_t a = first; a < arms; ++a)
        mbar_wait_one(full_bar(int(a % C::STAGES)), (a / C::STAGES) & 1u, 200000000ull);
    }
    __syncwarp();
  } else if (warp == 1 && !aborted_early) {
    // ------------------------------------------------------- MMA issuer
    bool ok = mbar_wait(tmem_ready_bar, 0, abort_flag, p.status, kStatusTimeoutMma);
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    int stage = 0;
    uint32_t phase = 0;
    int slot = 0;
    uint32_t sphase = 0;
    uint32_t lt = 0;
    int sfslot = 0;
    bool issued_any = false;
    while (ok) {
      if (!mbar_wait(schedf_bar(slot), sphase, abort_flag, p.status, kStatusTimeoutMma)) break;
      const uint32_t tile = sched_tile[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(schede_bar(slot));
      if (++slot == C::SCHED) {
        slot = 0;
        sphase ^= 1;
      }
      if (tile == kEndTile) break;
      const int g = int(tile >> 22);
      const int xti = int(tile & 0x7FFu);
      const int rows = tile_rows(g, xti);
      const int ncols = min(C::BN, (rows + 15) & ~15);
      const uint32_t b = lt & 1u;
      if (!mbar_wait(acce_bar(b), ((lt >> 1) & 1u) ^ 1u, abort_flag, p.status,
                     kStatusTimeoutMma))
        break;
      tc_fence_after();
      const uint32_t d_tmem = tmem + b * C::BN;
      for (int ks = 0; ks < p.ksteps; ++ks) {
        if (!mbar_wait(full_bar(stage), phase, abort_flag, p.status, kStatusTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint64_t adesc = desc_k_sw128(sW(stage));
          const uint64_t bdesc = desc_k_sw128(sX(stage));
          if constexpr (C::MX) {
            const uint32_t col = C::SF_BASE + sfslot * C::SF_SLOT;
            tc_cp_sf(tmem + col, desc_sf_atom(sSFW(stage)));
#pragma unroll
            for (int c = 0; c < C::CH; ++c)
              tc_cp_sf(tmem + col + 4 + 4 * c, desc_sf_atom(sSFX(stage) + c * 512));
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              // K step of 32 one-byte elements = 32 bytes = +2 in the start field;
              // SF id j picks byte j of every scale column.
              const uint32_t idesc =
                  idesc_block_scaled(kFmtF8E2M1, kFmtF8E4M3, 1, 128, ncols, j, j);
              tc_mma_mxf8f6f4(d_tmem, adesc + 2u * j, bdesc + 2u * j, idesc,
                              (tmem + col) | (uint32_t(j) << 30),
                              (tmem + col + 4) | (uint32_t(j) << 30), (ks | j) != 0 ? 1u : 0u);
            }
            sfslot = (sfslot + 1 == C::NSLOTS) ? 0 : sfslot + 1;
          } else {
            const uint32_t idesc =
                idesc_block_scaled(kFmtNvf4E2M1, kFmtNvf4E2M1, 0, 128, ncols, 0, 0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint32_t col = C::SF_BASE + sfslot * C::SF_SLOT;
              tc_cp_sf(tmem + col, desc_sf_atom(sSFW(stage) + j * 512));
#pragma unroll
              for (int c = 0; c < C::CH; ++c)
                tc_cp_sf(tmem + col + 4 + 4 * c,
                         desc_sf_atom(sSFX(stage) + (j * C::CH + c) * 512));
              // K step of 64 fp4 = 32 bytes = +2 in the descriptor's start field.
              tc_mma_nvf4(d_tmem, adesc + 2u * j, bdesc + 2u * j, idesc, tmem + col,
                          tmem + col + 4, (ks | j) != 0 ? 1u : 0u);
              sfslot = (sfslot + 1 == C::NSLOTS) ? 0 : sfslot + 1;
            }
          }
          tc_commit(empty_bar(stage));
        }
        __syncwarp();
        issued_any = true;
        if (++stage == C::STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
      if (!ok) break;
      if (lane == 0) tc_commit(accf_bar(b));
      __syncwarp();
      ++lt;
    }
    // Drain: every tcgen05 op this thread issued completes before TMEM is freed.
    if (lane == 0 && issued_any) {
      tc_commit(drain_bar);
      if (!mbar_wait_one(drain_bar, 0, 200000000ull)) atomicCAS(p.status, 0, kStatusTimeoutDrain);
    }
    __syncwarp();
  } else if (warp >= 4 && !aborted_early) {
    // --------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may read
    bool ok = mbar_wait(tmem_ready_bar, 0, abort_flag, p.status, kStatusTimeoutEpilogue);
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    int slot = 0;
    uint32_t sphase = 0;
    uint32_t lt = 0;
    while (ok) {
      if (!mbar_wait(schedf_bar(slot), sphase, abort_flag, p.status, kStatusTimeoutEpilogue))
        break;
      const uint32_t tile = sched_tile[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(schede_bar(slot));
      if (++slot == C::SCHED) {
        slot = 0;
        sphase ^= 1;
      }
      if (tile == kEndTile) break;
      const int g = int(tile >> 22);
      const int nti = int((tile >> 11) & 0x7FFu);
      const int xti = int(tile & 0x7FFu);
      const int rows = tile_rows(g, xti);
      const int ncols = min(C::BN, (rows + 15) & ~15);
      float alpha = 1.0f;
      size_t row0;
      if constexpr (C::MX) {
        row0 = size_t(xti) * C::BN;
      } else {
        alpha = p.alpha[g];
        row0 = size_t(p.ginfo[g].out_row) + size_t(xti) * C::BN;
      }
      const uint32_t b = lt & 1u;
      if (!mbar_wait(accf_bar(b), (lt >> 1) & 1u, abort_flag, p.status, kStatusTimeoutEpilogue))
        break;
      tc_fence_after();
      const int n = nti * 128 + q * 32 + lane;
      __nv_bfloat16* orow = p.out + row0 * size_t(p.n) + size_t(n);
      const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + b * C::BN;
      for (int c0 = 0; c0 < ncols; c0 += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + c0, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (c0 + j < rows)
            orow[size_t(c0 + j) * p.n] = __float2bfloat16_rn(alpha * __uint_as_float(r[j]));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar(b));
      ++lt;
    }
  }

  __syncthreads();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc(*tmem_holder, C::TMEM_COLS);
  }
  // The last CTA to finish rewinds the tile counter, so the next launch on the
  // same workspace (a replay without the prepare kernel) starts from tile 0.
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.status + 2, 1) == int(gridDim.x) - 1) {
      atomicExch(p.status + 1, 0);
      atomicExch(p.status + 2, 0);
    }
  }
}

// Set the kernel's dynamic shared memory limit (once per device), then launch
// one CTA per SM, or one per tile when there are fewer tiles.  Host only.
template <class C>
cudaError_t launch_engine(const GemmParams& gp, int sm_count, cudaStream_t s) {
  static int configured_device = -1;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (configured_device != dev) {
    e = cudaFuncSetAttribute(fgg_gemm_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(C::SMEM_BYTES));
    if (e != cudaSuccess) return e;
    configured_device = dev;
  }
  const int grid = gp.num_tiles < sm_count ? (gp.num_tiles > 0 ? gp.num_tiles : 1) : sm_count;
  fgg_gemm_kernel<C><<<grid, 256, C::SMEM_BYTES, s>>>(gp);
  return cudaGetLastError();
}

}  // namespace fgg
