// fgg_macro.cuh - the CTA-pair grouped GEMM with two token sub-tiles per
// weight tile.
//
// What bounds the pair kernel of fgg_engine.cuh on the grouped and dense
// shapes is the bytes its CTAs pull from L2 per K step (about 14 TB/s over
// the GPU), not the tensor pipe: every 224-token tile streams its CTA's 128
// weight rows (16 KB per K step) again.  This kernel takes a weight tile
// together with up to TWO consecutive 224-token tiles of the same group (a
// "macro tile") and issues each K step's MMAs for both against one copy of
// the weights: per CTA and K step 16 KB of weights serve 448 tokens instead
// of 224, about 25 % fewer L2 bytes per FLOP.
//
// TMEM: the two sub-tiles accumulate into the two 224-column regions that
// the pair kernel uses as a double buffer; a single-sub-tile tile (a group's
// last, odd token tile) takes one region, alternately, so a run of those is
// still double-buffered.  Regions are handed out in tile order by one rule
// that the MMA issuer and both epilogue groups evaluate alike:
//   single tile: region `next`, then next ^= 1
//   double tile: sub-tile A in `next`, B in `next ^ 1`
// Two epilogue warp groups (warps 4-7 and 8-11), one per region, drain the
// two sub-tiles of a double tile at the same time.  A double tile's MMAs wait
// for both regions to be drained, so its epilogue is not overlapped with the
// next double tile's MMAs the way a single tile's is; the two groups halve
// that wait.
//
// Everything else follows the pair kernel: warp 0 producer (both CTAs, TMA
// with .cta_group::2 completion on the leader's barrier, no multicast), warp
// 1 MMA issuer (leader), warp 2 TMEM allocator, warp 3 scheduler (leader,
// dynamic atomic tile counter, 8-deep slot ring published into both CTAs),
// every wait bounded.
#pragma once

#include "fgg_engine.cuh"

namespace fgg {

template <bool MX_, int STAGES_>
struct MacroCfg {
  static constexpr bool MX = MX_;
  static constexpr int BN = 224;   // tokens per sub-tile (MMA N at most)
  static constexpr int BNH = 112;  // token rows one CTA loads per sub-tile
  static constexpr int STAGES = STAGES_;
  static constexpr int KSUB = 1;
  static constexpr int K_STEP = MX ? 128 : 256;
  static constexpr uint32_t W_BYTES = 128 * 128;
  static constexpr uint32_t W_TX = MX ? 64 * 128 : 128 * 128;
  static constexpr uint32_t X_BYTES = BNH * 128;  // one sub-tile's half
  static constexpr uint32_t SFW_BYTES = MX ? 512 : 4 * 512;
  static constexpr uint32_t SFX_BYTES = MX ? 2 * 512 : 4 * 2 * 512;  // one sub-tile
  // SF atoms travel as 2-D uint64 boxes {ROW_U64, BOX_ROWS}, as in PairCfg
  static constexpr uint32_t SFW_ROW_U64 = SFW_BYTES / 8 > 256 ? 256 : SFW_BYTES / 8;
  static constexpr uint32_t SFW_BOX_ROWS = SFW_BYTES / (8 * SFW_ROW_U64);
  static constexpr uint32_t SFX_ROW_U64 = SFX_BYTES / 8 > 256 ? 256 : SFX_BYTES / 8;
  static constexpr uint32_t SFX_BOX_ROWS = SFX_BYTES / (8 * SFX_ROW_U64);
  static constexpr uint32_t TX_SINGLE = W_TX + X_BYTES + SFW_BYTES + SFX_BYTES;
  static constexpr uint32_t TX_DOUBLE = TX_SINGLE + X_BYTES + SFX_BYTES;
  // stage: [W | X_A | X_B] operand tiles, [SFW | SFX_A | SFX_B] atoms
  static constexpr uint32_t OP_BYTES = W_BYTES + 2 * X_BYTES;
  static constexpr uint32_t SF_BYTES = SFW_BYTES + 2 * SFX_BYTES;
  static constexpr uint32_t SUB_SLOTS = STAGES;
  static_assert(OP_BYTES % 1024 == 0, "operand tiles must stay 1024 B aligned");
  static_assert(SF_BYTES % 128 == 0, "scale atoms must stay 128 B aligned");
  // TMEM: regions [0, 224) and [224, 448); scale slots [weights 4 | A 8 | B 8]
  static constexpr int SF_BASE = 2 * BN;
  static constexpr int SF_SLOT = 20;
  static constexpr int NSLOTS = (512 - SF_BASE) / SF_SLOT;
  static_assert(NSLOTS >= 2, "not enough TMEM for the scale ring");
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int SCHED = 8;
  // readers of a slot: leader producer, MMA warp, 8 epilogue warps; follower
  // producer and 8 epilogue warps
  static constexpr uint32_t SCHED_READERS = 19;
  static constexpr int THREADS = 384;
  static constexpr uint32_t NBARS = 2 * STAGES + 4 + 2 * SCHED + 3;
  static constexpr uint32_t MISC_BYTES = 8 * NBARS + 32 * SCHED + 16;
  static constexpr uint32_t EPI_BYTES = 2 * kEpiStageBytes;  // 8 epilogue warps
  static constexpr uint32_t SF_REGION = SUB_SLOTS * OP_BYTES;
  static constexpr uint32_t BAR_REGION = SF_REGION + SUB_SLOTS * SF_BYTES;
  static constexpr uint32_t EPI_REGION = (BAR_REGION + MISC_BYTES + 15) / 16 * 16;
  static constexpr uint32_t SMEM_BYTES = 1024 + EPI_REGION + EPI_BYTES;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

// Metadata of macro tile `tile` = (group, weight tile, first token tile xt):
// sub-tile A is token tile xt, sub-tile B token tile xt + 1 when the group
// has it (pad[0] = B's rows, 0 for a single tile).
template <bool MX>
__device__ __forceinline__ SchedSlot make_macro_slot(const GemmParams& p, uint32_t tile) {
  SchedSlot s = make_slot<MX, 224>(p, tile);
  if (tile == kEndTile) return s;
  const int g = int(tile >> 22);
  const int xti = int(tile & 0x7FFu);
  int total;
  if constexpr (MX)
    total = p.m_total - xti * 224;  // MX macro tiles never cross an expert (see the tile list)
  else
    total = p.ginfo[g].m - xti * 224;
  s.pad[0] = max(0, min(224, total - 224));
  return s;
}

// Region use of a tile by the rule above: returns the region of sub-tile
// `sub` (0 = A, 1 = B) and advances `next` once per tile (call with sub 0).
__device__ __forceinline__ void macro_regions(bool dbl, uint32_t& next, uint32_t& ra,
                                              uint32_t& rb) {
  ra = next;
  rb = next ^ 1u;
  if (!dbl) next ^= 1u;
}

template <class C>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(384, 1)
    fgg_gemm_macro_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);

  const uint32_t bars = base + C::BAR_REGION;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (C::STAGES + s); };
  auto accf_bar = [&](uint32_t r) { return bars + 8u * (2 * C::STAGES + r); };
  auto acce_bar = [&](uint32_t r) { return bars + 8u * (2 * C::STAGES + 2 + r); };
  auto schedf_bar = [&](int i) { return bars + 8u * (2 * C::STAGES + 4 + i); };
  auto schede_bar = [&](int i) { return bars + 8u * (2 * C::STAGES + 4 + C::SCHED + i); };
  const uint32_t tmem_ready_bar = bars + 8u * (2 * C::STAGES + 4 + 2 * C::SCHED);
  const uint32_t drain_bar = tmem_ready_bar + 8u;
  const uint32_t taken_bar = tmem_ready_bar + 16u;
  uint8_t* const misc = gbase + C::BAR_REGION + 8 * C::NBARS;
  volatile SchedSlot* const ring = reinterpret_cast<volatile SchedSlot*>(misc);
  volatile uint32_t* const tmem_holder =
      reinterpret_cast<volatile uint32_t*>(misc + 32 * C::SCHED);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(misc + 32 * C::SCHED + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = (rank == 0);
  const uint32_t peer = rank ^ 1u;
  // epilogue warps 4-11: group (region) and TMEM lane quadrant
  const uint32_t egroup = uint32_t(warp >= 8 ? 1 : 0);
  uint32_t* const epi_stage = reinterpret_cast<uint32_t*>(
      gbase + C::EPI_REGION + ((warp - 4) & 7) * (kEpiStageBytes / 4));

  auto sW = [&](int q) { return base + q * C::OP_BYTES; };
  auto sX = [&](int q, int sub) { return base + q * C::OP_BYTES + C::W_BYTES + sub * C::X_BYTES; };
  auto sSFW = [&](int q) { return base + C::SF_REGION + q * C::SF_BYTES; };
  auto sSFX = [&](int q, int sub) {
    return base + C::SF_REGION + q * C::SF_BYTES + C::SFW_BYTES + sub * C::SFX_BYTES;
  };
  auto tile_ncols = [&](int rows) -> int { return min(C::BN, (rows + 31) & ~31); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (uint32_t r = 0; r < 2; ++r) {
      mbar_init(accf_bar(r), 1);
      mbar_init(acce_bar(r), 8);  // the region's 4 epilogue warps in each CTA
    }
    for (int i = 0; i < C::SCHED; ++i) {
      mbar_init(schedf_bar(i), 1);
      mbar_init(schede_bar(i), C::SCHED_READERS);
    }
    mbar_init(tmem_ready_bar, 1);
    mbar_init(drain_bar, 1);
    mbar_init(taken_bar, 1);
    *abort_flag = 0;
    if constexpr (!C::MX) {
      const PackHeader h = *p.pack;
      if (h.magic != kPackMagic || h.g != p.wg || h.n != p.n || h.k != p.k) *abort_flag = 2;
    }
    fence_mbar_init();
  }
  cluster_sync();

  if (warp == 2) {
    tmem_alloc_pair(smem_u32(const_cast<uint32_t*>(tmem_holder)), C::TMEM_COLS);
    tmem_relinquish_pair();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(tmem_ready_bar);
  }

  griddep_wait();
  const bool aborted_early = (*abort_flag != 0);
  if (threadIdx.x == 0 && *abort_flag == 2) atomicCAS(p.status, 0, kStatusBadPack);
  const uint32_t leader_schede0 = mapa_shared(schede_bar(0), 0);
  const uint32_t leader_acce0 = mapa_shared(acce_bar(0), 0);
  const uint32_t leader_full0 = mapa_shared(full_bar(0), 0);

  auto release_slot = [&](int slot) {
    if (leader)
      mbar_arrive(schede_bar(slot));
    else
      mbar_arrive_remote(leader_schede0 + 8u * slot);
  };

  if (warp == 3) {
    // ---------------------------------------------- scheduler (leader only)
    if (lane == 0 && leader && !aborted_early) {
      int slot = 0;
      uint32_t sphase = 0;
      const int num_tiles = p.num_tiles_dev != nullptr ? *p.num_tiles_dev : p.num_tiles;
      const uint32_t remote_ring0 = mapa_shared(smem_u32(const_cast<SchedSlot*>(ring)), peer);
      const uint32_t remote_schedf0 = mapa_shared(schedf_bar(0), peer);
      for (uint32_t n = 0;; ++n) {
        if (n > 0 && !mbar_wait1(taken_bar, (n - 1) & 1u, abort_flag, p.status,
                                 kStatusTimeoutProducer))
          break;
        const int t = atomicAdd(p.status + 1, 1);
        const uint32_t tile = (t < num_tiles) ? __ldg(p.tiles + t) : kEndTile;
        const SchedSlot s = make_macro_slot<C::MX>(p, tile);
        if (!mbar_wait1<true>(schede_bar(slot), sphase ^ 1, abort_flag, p.status,
                              kStatusTimeoutProducer))
          break;
        write_slot(ring, slot, s);
        ring[slot].pad[0] = s.pad[0];
        write_slot_remote(remote_ring0, slot, s);
        mbar_arrive(schedf_bar(slot));
        mbar_arrive_remote(remote_schedf0 + 8u * slot);
        if (++slot == C::SCHED) {
          slot = 0;
          sphase ^= 1;
        }
        if (tile == kEndTile) break;
      }
    }
    __syncwarp();
  } else if (warp == 0) {
    // ------------------------------------------------- producer (both CTAs)
    if (!aborted_early) {
      int stage = 0;
      uint32_t phase = 0;
      int slot = 0;
      uint32_t sphase = 0;
      uint32_t arms = 0;
      if (lane == 0) {
        if constexpr (C::MX) prefetch_tensormap(&p.mx_tmap_w);
        if (C::MX || p.x_flat) prefetch_tensormap(&p.tmap_x_flat);
        prefetch_tensormap(&p.sfw_map);
        prefetch_tensormap(&p.sfx_map);
      }
      while (true) {
        if (!mbar_wait<true>(schedf_bar(slot), sphase, abort_flag, p.status,
                             kStatusTimeoutProducer))
          break;
        const uint32_t tile = __shfl_sync(kFullMask, ring[slot].tile, 0);
        const int rows_a = __shfl_sync(kFullMask, ring[slot].rows, 0);
        const int rows_b = __shfl_sync(kFullMask, ring[slot].pad[0], 0);
        const int xtile_index = __shfl_sync(kFullMask, ring[slot].xtile_index, 0);
        const int wgroup = __shfl_sync(kFullMask, ring[slot].wgroup, 0);
        const int row0 = __shfl_sync(kFullMask, ring[slot].row0, 0);
        if (lane == 0) {
          release_slot(slot);
          if (leader) mbar_arrive(taken_bar);
        }
        if (++slot == C::SCHED) {
          slot = 0;
          sphase ^= 1;
        }
        if (tile == kEndTile) {
          if (lane == 0) griddep_launch_dependents();
          break;
        }
        const int g = int(tile >> 22);
        const int nti = int((tile >> 11) & 0x7FFu);
        const int xti = int(tile & 0x7FFu);
        if (g >= p.g || unsigned(wgroup) >= unsigned(p.wg)) {
          if (lane == 0) {
            atomicCAS(p.status, 0, kStatusBadTile);
            *abort_flag = 1;
          }
          break;
        }
        const bool dbl = rows_b > 0;
        const int half_a = tile_ncols(rows_a) >> 1;
        const int half_b = tile_ncols(rows_b) >> 1;
        const CUtensorMap* tw;
        const CUtensorMap* tx;
        if constexpr (C::MX) {
          tw = &p.mx_tmap_w;
          tx = &p.tmap_x_flat;
        } else {
          tw = p.tmap_w + wgroup;
          tensormap_acquire(tw);
          if (p.x_flat) {
            tx = &p.tmap_x_flat;
          } else {
            tx = p.tmap_x + g;
            tensormap_acquire(tx);
          }
        }
        const int wrow = nti * 256 + int(rank) * 128;
        // the two sub-tiles' first token rows in the map's coordinates
        const int xbase = (C::MX || p.x_flat) ? row0 : xti * C::BN;
        const int xrow_a = xbase + int(rank) * half_a;
        const int xrow_b = xbase + C::BN + int(rank) * half_b;
        const int sfw_y =
            ((wgroup * p.nt128 + 2 * nti + int(rank)) * p.ksteps) * int(C::SFW_BOX_ROWS);
        const int sfx_y = (xtile_index * p.ksteps) * int(C::SFX_BOX_ROWS);
        const int sfx_y_b = ((xtile_index + 1) * p.ksteps) * int(C::SFX_BOX_ROWS);
        const uint32_t tx_bytes = 2u * (dbl ? C::TX_DOUBLE : C::TX_SINGLE);
        bool ok = true;
        for (int ks = 0; ks < p.ksteps; ++ks) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.status,
                         kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = leader_full0 + 8u * stage;
          const bool arm = (p.debug_flags & kDebugNoLoads) == 0;
          if (arm && elect_one()) {
            if (leader) mbar_arrive_expect_tx(full_bar(stage), tx_bytes);
            if constexpr (C::MX)
              tma_load_3d_pair(sW(stage), tw, fb, ks * C::K_STEP, wrow, g);
            else
              tma_load_2d_pair(sW(stage), tw, fb, ks * 128, wrow);
            tma_load_2d_pair(sX(stage, 0), tx, fb, ks * 128, xrow_a);
            tma_load_2d_pair(sSFW(stage), &p.sfw_map, fb, 0, sfw_y + ks * int(C::SFW_BOX_ROWS));
            tma_load_2d_pair(sSFX(stage, 0), &p.sfx_map, fb, 0, sfx_y + ks * int(C::SFX_BOX_ROWS));
            if (dbl) {
              tma_load_2d_pair(sX(stage, 1), tx, fb, ks * 128, xrow_b);
              tma_load_2d_pair(sSFX(stage, 1), &p.sfx_map, fb, 0,
                               sfx_y_b + ks * int(C::SFX_BOX_ROWS));
            }
          }
          __syncwarp();
          if (arm) ++arms;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
      }
      if (leader && lane == 0) {
        const uint32_t first = arms > uint32_t(C::STAGES) ? arms - C::STAGES : 0u;
        for (uint32_t a = first; a < arms; ++a)
          mbar_wait_one(full_bar(int(a % C::STAGES)), (a / C::STAGES) & 1u, 200000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1 && leader) {
    // ------------------------------------------------------- MMA issuer
    if (!aborted_early) {
      bool ok = mbar_wait(tmem_ready_bar, 0, abort_flag, p.status, kStatusTimeoutMma);
      tc_fence_after();
      const uint32_t tmem = __shfl_sync(kFullMask, *tmem_holder, 0);
      int stage = 0;
      uint32_t phase = 0;
      int slot = 0;
      uint32_t sphase = 0;
      uint32_t next = 0;
      uint32_t uses[2] = {0u, 0u};
      int sfslot = 0;
      bool issued_any = false;
      while (ok) {
        if (!mbar_wait<true>(schedf_bar(slot), sphase, abort_flag, p.status, kStatusTimeoutMma))
          break;
        const uint32_t tile = __shfl_sync(kFullMask, ring[slot].tile, 0);
        const int rows_a = __shfl_sync(kFullMask, ring[slot].rows, 0);
        const int rows_b = __shfl_sync(kFullMask, ring[slot].pad[0], 0);
        if (lane == 0) mbar_arrive(schede_bar(slot));
        if (++slot == C::SCHED) {
          slot = 0;
          sphase ^= 1;
        }
        if (tile == kEndTile) break;
        const bool dbl = rows_b > 0;
        uint32_t ra, rb;
        macro_regions(dbl, next, ra, rb);
        // the regions this tile writes must be drained by their epilogue group
        if (!mbar_wait(acce_bar(ra), (uses[ra] & 1u) ^ 1u, abort_flag, p.status,
                       kStatusTimeoutMma))
          break;
        if (dbl && !mbar_wait(acce_bar(rb), (uses[rb] & 1u) ^ 1u, abort_flag, p.status,
                              kStatusTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d_a = tmem + ra * C::BN;
        const uint32_t d_b = tmem + rb * C::BN;
        const int ncols_a = tile_ncols(rows_a);
        const int ncols_b = dbl ? tile_ncols(rows_b) : 32;
        const uint32_t idesc_a =
            C::MX ? 0u : idesc_block_scaled(kFmtNvf4E2M1, kFmtNvf4E2M1, 0, 256, ncols_a, 0, 0);
        const uint32_t idesc_b =
            C::MX ? 0u : idesc_block_scaled(kFmtNvf4E2M1, kFmtNvf4E2M1, 0, 256, ncols_b, 0, 0);
        for (int ks = 0; ks < p.ksteps; ++ks) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, p.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          constexpr int kSlots = C::MX ? 1 : 4;
          uint32_t col[kSlots];
#pragma unroll
          for (int i = 0; i < kSlots; ++i) {
            col[i] = tmem + C::SF_BASE + sfslot * C::SF_SLOT;
            sfslot = (sfslot + 1 == C::NSLOTS) ? 0 : sfslot + 1;
          }
          const bool last = ks + 1 == p.ksteps;
          if (elect_one()) {
            const uint64_t adesc = desc_k_sw128(sW(stage));
            const uint64_t bdesc_a = desc_k_sw128(sX(stage, 0));
            const uint64_t bdesc_b = desc_k_sw128(sX(stage, 1));
            if constexpr (C::MX) {
              const uint32_t c0 = col[0];
              tc_cp_sf_pair(c0, desc_sf_atom(sSFW(stage)));
              tc_cp_sf_pair(c0 + 4, desc_sf_atom(sSFX(stage, 0)));
              tc_cp_sf_pair(c0 + 8, desc_sf_atom(sSFX(stage, 0) + 512));
              if (dbl) {
                tc_cp_sf_pair(c0 + 12, desc_sf_atom(sSFX(stage, 1)));
                tc_cp_sf_pair(c0 + 16, desc_sf_atom(sSFX(stage, 1) + 512));
              }
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t acc = (ks | j) != 0 ? 1u : 0u;
                const uint32_t sfa = c0 | (uint32_t(j) << 30);
                tc_mma_mxf8f6f4_pair(d_a, adesc + 2u * j, bdesc_a + 2u * j,
                                     idesc_block_scaled(kFmtF8E2M1, kFmtF8E4M3, 1, 256, ncols_a, j, j),
                                     sfa, (c0 + 4) | (uint32_t(j) << 30), acc);
                if (dbl)
                  tc_mma_mxf8f6f4_pair(d_b, adesc + 2u * j, bdesc_b + 2u * j,
                                       idesc_block_scaled(kFmtF8E2M1, kFmtF8E4M3, 1, 256, ncols_b, j, j),
                                       sfa, (c0 + 12) | (uint32_t(j) << 30), acc);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t c0 = col[j];
                const uint32_t acc = (ks | j) != 0 ? 1u : 0u;
                tc_cp_sf_pair(c0, desc_sf_atom(sSFW(stage) + j * 512));
                tc_cp_sf_pair(c0 + 4, desc_sf_atom(sSFX(stage, 0) + (2 * j) * 512));
                tc_cp_sf_pair(c0 + 8, desc_sf_atom(sSFX(stage, 0) + (2 * j + 1) * 512));
                if (dbl) {
                  tc_cp_sf_pair(c0 + 12, desc_sf_atom(sSFX(stage, 1) + (2 * j) * 512));
                  tc_cp_sf_pair(c0 + 16, desc_sf_atom(sSFX(stage, 1) + (2 * j + 1) * 512));
                }
                tc_mma_nvf4_pair(d_a, adesc + 2u * j, bdesc_a + 2u * j, idesc_a, c0, c0 + 4, acc);
                if (dbl)
                  tc_mma_nvf4_pair(d_b, adesc + 2u * j, bdesc_b + 2u * j, idesc_b, c0, c0 + 12,
                                   acc);
              }
            }
            tc_commit_pair(empty_bar(stage), 0x3);
            if (last) {
              tc_commit_pair(accf_bar(ra), 0x3);
              if (dbl) tc_commit_pair(accf_bar(rb), 0x3);
            }
          }
          __syncwarp();
          issued_any = true;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ++uses[ra];
        if (dbl) ++uses[rb];
      }
      if (issued_any) {
        if (elect_one()) {
          tc_commit_pair(drain_bar, 0x1);
          if (!mbar_wait_one(drain_bar, 0, 200000000ull))
            atomicCAS(p.status, 0, kStatusTimeoutDrain);
        }
      }
    }
    __syncwarp();
  } else if (warp >= 4 && !aborted_early) {
    // --------------------------------------------------------- epilogue
    // group `egroup` drains region `egroup`
    const int q = warp & 3;
    bool ok = mbar_wait(tmem_ready_bar, 0, abort_flag, p.status, kStatusTimeoutEpilogue);
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    int slot = 0;
    uint32_t sphase = 0;
    uint32_t next = 0;
    uint32_t uses = 0;
    while (ok) {
      if (!mbar_wait<true>(schedf_bar(slot), sphase, abort_flag, p.status,
                           kStatusTimeoutEpilogue))
        break;
      const SchedSlot s = read_slot(ring, slot);
      const int rows_b = ring[slot].pad[0];
      __syncwarp();
      if (lane == 0) release_slot(slot);
      if (++slot == C::SCHED) {
        slot = 0;
        sphase ^= 1;
      }
      if (s.tile == kEndTile) break;
      const bool dbl = rows_b > 0;
      uint32_t ra, rb;
      macro_regions(dbl, next, ra, rb);
      int sub = -1;
      if (ra == egroup) sub = 0;
      else if (dbl && rb == egroup) sub = 1;
      if (sub < 0) continue;  // the other group's region
      const int nti = int((s.tile >> 11) & 0x7FFu);
      const int rows = sub == 0 ? s.rows : rows_b;
      const int ncols = tile_ncols(rows);
      if (!mbar_wait(accf_bar(egroup), uses & 1u, abort_flag, p.status, kStatusTimeoutEpilogue))
        break;
      tc_fence_after();
      const size_t row0 = size_t(s.row0) + size_t(sub * C::BN);
      const uint32_t taddr = tmem + (uint32_t(q * 32) << 16) + egroup * C::BN;
      if (p.epi == kEpiSiluMul)
        epilogue_tile_silu_mul(p.out, p.n / 2, nti * 256 + int(rank) * 128 + q * 32, row0, rows,
                               ncols, s.alpha, taddr);
      else
        epilogue_tile(p.out, p.n, nti * 256 + int(rank) * 128 + q * 32, row0, rows, ncols,
                      s.alpha, p.row_scale, taddr, epi_stage);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(acce_bar(egroup));
        else
          mbar_arrive_remote(leader_acce0 + 8u * egroup);
      }
      ++uses;
    }
  }

  __syncthreads();
  cluster_sync();
  if (warp == 2) {
    tc_fence_after();
    tmem_dealloc_pair(*tmem_holder, C::TMEM_COLS);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.status + 2, 1) == int(gridDim.x) - 1) {
      atomicExch(p.status + 1, 0);
      atomicExch(p.status + 2, 0);
    }
  }
}

// One CTA pair per two SMs (384 threads each), or one per tile when there are
// fewer tiles.  Host only.
template <class C>
cudaError_t launch_macro(const GemmParams& gp, int sm_count, cudaStream_t s) {
  if (ensure_max_dynamic_smem(reinterpret_cast<const void*>(fgg_gemm_macro_kernel<C>),
                              int(C::SMEM_BYTES)) != FGG_OK)
    return cudaErrorInvalidValue;
  const int pairs_avail = sm_count / 2;
  const int pairs = gp.num_tiles < pairs_avail ? (gp.num_tiles > 0 ? gp.num_tiles : 1) : pairs_avail;
  return launch_pdl(fgg_gemm_macro_kernel<C>, dim3(unsigned(2 * pairs)), dim3(C::THREADS),
                    C::SMEM_BYTES, s, gp);
}

}  // namespace fgg
