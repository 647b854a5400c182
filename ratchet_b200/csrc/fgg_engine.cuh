// fgg_engine.cuh - the persistent tcgen05 grouped-GEMM engine shared by both
// operand formats.
//
// Orientation ("swap AB", as kernels/gemm/fp4_grouped_gemm/b200/kernel.py:84-86
// does with MMA-A = weights): the tensor core's M axis runs over weight rows
// (output columns n), its N axis over up to BN tokens of one group (output rows
// m).  Ragged group sizes land on the MMA's N axis, sized per tile in steps of
// 16 (32 for pairs), and the epilogue's lanes walk consecutive output columns.
//
// Warp roles (256 threads, one CTA per SM):
//   warp 0     producer: the TMA loads of every K step into a STAGES-deep
//              shared-memory ring
//   warp 1     MMA issuer: tcgen05.cp (scale factors -> TMEM) and the
//              block-scaled tcgen05.mma chain into a double-buffered TMEM
//              accumulator
//   warp 2     TMEM allocator
//   warp 3     scheduler: claims tiles from a global atomic counter (dynamic
//              persistent schedule) and publishes each tile with its metadata
//              in an 8-deep shared-memory ring, one tile ahead of the
//              producer (the ring's depth covers the roles that lag behind)
//   warps 4-7  epilogue: tcgen05.ld (each warp its 32-lane quadrant) -> fp32
//              x alpha -> bf16 -> global (or the gated SiLU * up form),
//              overlapped with the next tile's MMAs
// The producer and MMA roles run their loops on the whole warp, so that every
// operand of a TMA or tcgen05 instruction (smem descriptors, TMEM columns,
// coordinates) is computed warp-uniformly, and issue from one elect.sync
// region per stage.  Issued that way a 32x128b.warpx4 scale copy costs the
// issuing thread under 10 cycles; from a lone lane with per-thread operands
// each TMA or tcgen05 instruction held it for 45-60, which bounded the kernel.
// Scale factors therefore travel as plain 512-byte atoms, one small copy each
// (a 128x256b copy would take one instruction for two atoms, but costs the
// tensor pipe 50-64 cycles that do not overlap the MMAs).  Every wait
// suspends in hardware (try_wait with a time hint) so waiting warps do not
// steal issue slots, and the epilogue keeps its instruction stream short for
// the same reason.
//
// Two kernels:
//   fgg_gemm_kernel       one CTA per tile, 128 weight rows x BN tokens
//   fgg_gemm_pair_kernel  a CTA pair (cta_group::2) per tile, 256 x 224: each
//                         CTA loads half of the token tile
// Two kinds (compile-time):
//   NVFP4   .kind::mxf4nvf4 .scale_vec::4X: E2M1 x E2M1, one E4M3 scale per 16
//           K; K step 256 = 4 MMAs of K 64, one SF slot per MMA.
//   MX      .kind::mxf8f6f4: weights E2M1 (4-bit codes unpacked to bytes by
//           TMA), tokens E4M3, one UE8M0 scale per 32 K; K step 128 = 4 MMAs of
//           K 32 that share one SF slot and pick their byte with the SF id.
#pragma once

#include <cuda_bf16.h>

#include "fgg_host.cuh"
#include "fgg_ptx.cuh"

namespace fgg {

struct GroupInfo {
  int32_t m;            // rows of A_g
  int32_t out_row;      // first output row of the group
  int32_t xtile_begin;  // index of the group's first token tile in the SF repack
  int32_t wgroup;       // weight group (in the pack) this problem group multiplies with
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
constexpr int kStatusBadTile = 0x202;  // a schedule slot named a group outside the problem

// One schedule-ring slot (32 bytes): what every role needs to know about a
// tile, published by the scheduler warp.
struct SchedSlot {
  uint32_t tile;        // packed (group, weight tile, token tile) or kEndTile
  int32_t rows;         // valid token rows of the tile
  int32_t row0;         // output row of the tile's first token
  float alpha;          // output scale
  int32_t xtile_index;  // the token tile's index in the token-scale repack
  int32_t wgroup;       // weight group of the tile (NVFP4 pack index; MX expert)
  int32_t pad[2];
};
static_assert(sizeof(SchedSlot) == 32, "slot is 8 words");

// Narrow token boxes of the pair kernel: 16, 32, ..., 16 * kXSmallMaps rows.
constexpr int kXSmallMaps = 6;

struct GemmParams {
  CUtensorMap mx_tmap_w;      // MX: 3-D map of the [G, N, K] weight codes
  // One 2-D map over contiguous token rows: MX [M_total, K] fp8 activations;
  // NVFP4 with x_flat set: [max_rows, K/2] codes of every group
  CUtensorMap tmap_x_flat;
  CUtensorMap sfw_map;        // pair kernel: the weight SF atoms as a 2-D uint64 tensor
  CUtensorMap sfx_map;        // pair kernel: the token SF atoms as a 2-D uint64 tensor
  // pair kernel, NVFP4 with x_flat and x_small set: maps over the same token
  // rows as tmap_x_flat with boxes of 16, 32, ..., 96 rows, so that a tile
  // whose MMA is narrower than 224 columns loads only the rows it uses
  CUtensorMap tmap_x_small[kXSmallMaps];
  const CUtensorMap* tmap_w;  // NVFP4: [G] per-group maps (global memory)
  const CUtensorMap* tmap_x;  // NVFP4: [G] per-group maps (global memory)
  const uint8_t* sfw;         // [G][NT128][KSTEPS][SFW_BYTES]
  const uint8_t* sfx;         // [XT][KSTEPS][SFX_BYTES]
  const GroupInfo* ginfo;     // NVFP4: [G]
  const uint32_t* tiles;      // [T]
  const float* alpha;         // NVFP4: [G]; MX: unused (1)
  const PackHeader* pack;     // NVFP4: weight pack header; MX: null
  __nv_bfloat16* out;
  int* status;  // [0] status, [1] tile counter, [2] finished CTAs
  int32_t g, n, k;
  int32_t wg;       // NVFP4: weight groups in the pack (problem groups index into it)
  int32_t m_total;  // MX: rows of the contiguous activation tensor
  int32_t num_tiles;
  int32_t ksteps;
  int32_t nt;     // weight tiles per group in the tile list (128 rows; 256 for pairs)
  int32_t nt128;  // 128-row weight tiles per group (the SF pack's unit)
  int32_t epi;    // kEpiPlain or kEpiSiluMul (NVFP4 only)
  int32_t debug_flags;  // test hooks (kDebugNoLoads); 0 in normal use
  // NVFP4: 1 = the token rows of all groups lie in one buffer read through
  // tmap_x_flat, the tile's first row being its output row (group offsets
  // from the device); 0 = one descriptor per group (tmap_x)
  int32_t x_flat;
  // optional device [rows] factor per output row (token), applied with alpha:
  // out[t, n] = bf16(alpha_g * row_scale[t] * acc); null = 1
  const float* row_scale;
  // optional device word holding the tile count (written by the prepare
  // kernel); null = num_tiles
  const int32_t* num_tiles_dev;
  int32_t x_small;  // 1: tmap_x_small is encoded (x_flat only)
};

// Test hook: the producer arms no stage and issues no load, so the MMA role's
// wait on the first full barrier runs out (a barrier nothing completes) and the
// kernel ends through its bounded-wait path with a non-zero status word.
constexpr int32_t kDebugNoLoads = 1;

// Epilogues.  kEpiPlain: out[t, n] = bf16(alpha * acc).  kEpiSiluMul: the
// weight rows come in 32-row chunks of 16 gate rows then the 16 up rows of the
// same outputs; out[t, 16c + i] = bf16(silu(alpha * gate) * (alpha * up)) with
// row stride N/2.
constexpr int32_t kEpiPlain = 0;
constexpr int32_t kEpiSiluMul = 1;

// Metadata of tile `tile` (scheduler warp, off the critical path).
template <bool MX, int BN>
__device__ __forceinline__ SchedSlot make_slot(const GemmParams& p, uint32_t tile) {
  SchedSlot s;
  s.tile = tile;
  s.pad[0] = s.pad[1] = 0;
  if (tile == kEndTile) {
    s.rows = 0;
    s.row0 = 0;
    s.alpha = 0.0f;
    s.xtile_index = 0;
    s.wgroup = 0;
    return s;
  }
  const int g = int(tile >> 22);
  const int xti = int(tile & 0x7FFu);
  if constexpr (MX) {
    s.rows = min(BN, p.m_total - xti * BN);
    s.row0 = xti * BN;
    s.alpha = 1.0f;
    s.xtile_index = xti;
    s.wgroup = g;
  } else {
    const GroupInfo gi = p.ginfo[g];
    s.rows = min(BN, gi.m - xti * BN);
    s.row0 = gi.out_row + xti * BN;
    s.alpha = p.alpha[g];
    s.xtile_index = gi.xtile_begin + xti;
    s.wgroup = gi.wgroup;
  }
  return s;
}

__device__ __forceinline__ SchedSlot read_slot(const volatile SchedSlot* ring, int slot) {
  SchedSlot s;
  s.tile = ring[slot].tile;
  s.rows = ring[slot].rows;
  s.row0 = ring[slot].row0;
  s.alpha = ring[slot].alpha;
  s.xtile_index = ring[slot].xtile_index;
  s.wgroup = ring[slot].wgroup;
  return s;
}

// Publish a slot into the peer CTA's ring (cluster address of its slot 0):
// every 32-bit word of the slot, so no field can be left stale in the peer.
__device__ __forceinline__ void write_slot_remote(uint32_t remote_ring0, int slot,
                                                  const SchedSlot& s) {
  const uint32_t words[8] = {s.tile,
                             uint32_t(s.rows),
                             uint32_t(s.row0),
                             __float_as_uint(s.alpha),
                             uint32_t(s.xtile_index),
                             uint32_t(s.wgroup),
                             uint32_t(s.pad[0]),
                             uint32_t(s.pad[1])};
  static_assert(sizeof(SchedSlot) == sizeof(words), "every word of the slot is stored");
#pragma unroll
  for (int i = 0; i < 8; ++i) st_shared_remote_u32(remote_ring0 + 32u * slot + 4u * i, words[i]);
}

__device__ __forceinline__ void write_slot(volatile SchedSlot* ring, int slot,
                                           const SchedSlot& s) {
  ring[slot].tile = s.tile;
  ring[slot].rows = s.rows;
  ring[slot].row0 = s.row0;
  ring[slot].alpha = s.alpha;
  ring[slot].xtile_index = s.xtile_index;
  ring[slot].wgroup = s.wgroup;
}

// Shared-memory staging of the plain epilogue: 16 tokens x 16 words (32 bf16
// output columns) per epilogue warp.
constexpr uint32_t kEpiStageBytes = 4 * 16 * 16 * 4;

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Epilogue of one tile for the calling warp: its 32 TMEM lanes are the
// output columns n0 + lane, its TMEM columns the tile's tokens.  Per 16
// tokens: one tcgen05.ld (lane = column, register j = token), x alpha (x the
// token's row scale), then a transpose through the warp's 1 KB staging area so
// that every lane stores 16 contiguous bytes -- 8 columns of one token row --
// instead of 16 scattered 2-byte values:
//   * token pairs (j, j+1): one shuffle across neighbouring lanes gives the
//     even lane columns (l, l+1) of token j and the odd lane the same columns
//     of token j+1; each stores that word at [token][column pair] (the two
//     rows of a pair land in opposite bank halves: conflict-free);
//   * each lane reads back 16 bytes (token lane/4, then lane/4 + 8; columns
//     8 (lane % 4) .. +7) and stores them to global memory.
// A row scale, when given, comes one value per lane (lanes 0-15) and is
// broadcast by shuffles.  Rows past `rows` are neither scaled nor stored.
__device__ __forceinline__ void epilogue_tile(__nv_bfloat16* out, int ldn, int n0, size_t row0,
                                              int rows, int ncols, float alpha,
                                              const float* __restrict__ row_scale, uint32_t taddr,
                                              uint32_t* stage) {
  const int lane = threadIdx.x & 31;
  const bool odd = lane & 1;
  for (int c0 = 0; c0 < ncols; c0 += 16) {
    uint32_t r[16];
    tmem_ld16(taddr + c0, r);
    float rs = 1.0f;
    if (row_scale != nullptr && lane < 16 && c0 + lane < rows)
      rs = __ldg(row_scale + row0 + size_t(c0 + lane));
    tmem_wait_ld();
    float v[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      v[j] = alpha * __uint_as_float(r[j]);
      if (row_scale != nullptr) v[j] *= __shfl_sync(kFullMask, rs, j);
    }
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const float got = __shfl_xor_sync(kFullMask, odd ? v[j] : v[j + 1], 1);
      const uint32_t w = odd ? pack_bf16x2(got, v[j + 1]) : pack_bf16x2(v[j], got);
      stage[(j + (odd ? 1 : 0)) * 16 + (lane >> 1)] = w;
    }
    __syncwarp();
    const int seg = lane & 3;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int t = (lane >> 2) + 8 * h;
      const uint4 q = *reinterpret_cast<const uint4*>(stage + t * 16 + 4 * seg);
      if (c0 + t < rows)
        *reinterpret_cast<uint4*>(out + (row0 + size_t(c0 + t)) * size_t(ldn) + size_t(n0 + 8 * seg)) = q;
    }
    __syncwarp();
  }
}

// Gated epilogue of one tile for the calling warp (kEpiSiluMul): lanes 0-15
// hold 16 gate rows, lanes 16-31 the up rows of the same 16 outputs.  Two
// token columns at a time: one shuffle across the half-warps gives lanes 0-15
// the up values of column j and lanes 16-31 the gate values of column j + 1,
// so every lane computes one silu(gate) * up (silu(x) = x * sigmoid(x),
// sigmoid(x) = (1 + tanh(x / 2)) / 2 on the hardware tanh).  n0: the warp's
// first weight row (a multiple of 32); out has N/2 columns.
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void epilogue_tile_silu_mul(__nv_bfloat16* out, int ldn_half, int n0,
                                                       size_t row0, int rows, int ncols,
                                                       float alpha, uint32_t taddr) {
  const int lane = threadIdx.x & 31;
  const bool gate_half = lane < 16;
  __nv_bfloat16* ocol = out + row0 * size_t(ldn_half) + size_t(n0 / 2 + (lane & 15));
  for (int c0 = 0; c0 < ncols; c0 += 16) {
    uint32_t r[16];
    tmem_ld16(taddr + c0, r);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const float v0 = alpha * __uint_as_float(r[j]);
      const float v1 = alpha * __uint_as_float(r[j + 1]);
      const float got = __shfl_xor_sync(0xffffffffu, gate_half ? v1 : v0, 16);
      const float g = gate_half ? v0 : got;
      const float u = gate_half ? got : v1;
      const float h = g * fmaf(0.5f, tanh_approx(0.5f * g), 0.5f) * u;
      const int t = c0 + j + (gate_half ? 0 : 1);
      if (t < rows) ocol[size_t(t) * ldn_half] = __float2bfloat16_rn(h);
    }
  }
}

template <bool MX_, int BN_, int STAGES_, int KSUB_ = 1>
struct EngineCfg {
  static constexpr bool MX = MX_;
  static constexpr int BN = BN_;
  static constexpr int STAGES = STAGES_;
  // K steps per pipeline stage (one barrier wait and one commit per stage)
  static constexpr int KSUB = KSUB_;
  static_assert(KSUB == 1 || KSUB == 2, "one or two K steps per stage");
  static constexpr int CH = (BN + 127) / 128;  // 128-row SF atoms per token tile
  // K elements per pipeline stage: one 128-byte swizzle row of each operand.
  static constexpr int K_STEP = MX ? 128 : 256;
  static constexpr uint32_t W_BYTES = 128 * 128;   // smem bytes of the weight tile
  static constexpr uint32_t W_TX = MX ? 64 * 128 : 128 * 128;  // bytes TMA reads from HBM
  static constexpr uint32_t X_BYTES = BN * 128;
  // NVFP4: 4 atoms (one per K64 MMA); MX: one atom covers the 4 K32 MMAs.
  static constexpr uint32_t SFW_BYTES = MX ? 512 : 4 * 512;
  // token scales: CH atoms per MMA (NVFP4) or per K step (MX)
  static constexpr uint32_t SFX_BYTES = MX ? CH * 512 : 4 * CH * 512;
  static constexpr uint32_t TX_BYTES = W_TX + X_BYTES + SFW_BYTES + SFX_BYTES;
  // Shared memory of one K step: its two operand tiles (1024 B aligned for
  // the 128-byte swizzle) in one region, its scale atoms in another, so that
  // no stage pads its atoms up to a 1024-byte boundary.  A stage holds KSUB
  // K steps.
  static constexpr uint32_t OP_BYTES = W_BYTES + X_BYTES;
  static constexpr uint32_t SF_BYTES = SFW_BYTES + SFX_BYTES;
  static constexpr uint32_t SUB_SLOTS = STAGES_ * KSUB;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "BN must be a multiple of 16");
  static_assert(OP_BYTES % 1024 == 0, "operand tiles must stay 1024 B aligned");
  static_assert(SF_BYTES % 128 == 0, "scale atoms must stay 128 B aligned");
  // TMEM columns: two accumulators of BN fp32 columns, then a ring of scale
  // slots (4 columns of weight scales + 4 per token atom).  NVFP4 takes one
  // slot per MMA, MX one per K step.
  static constexpr int SF_BASE = ((2 * BN + 3) / 4) * 4;
  static constexpr int SF_SLOT = 4 + 4 * CH;
  static constexpr int NSLOTS_FIT = (512 - SF_BASE) / SF_SLOT;
  static constexpr int NSLOTS = NSLOTS_FIT > 8 ? 8 : NSLOTS_FIT;
  static_assert(NSLOTS >= 2, "not enough TMEM for the scale ring");
  static constexpr int COLS = SF_BASE + NSLOTS * SF_SLOT;
  static_assert(COLS <= 512, "TMEM columns exceeded");
  static constexpr uint32_t TMEM_COLS =
      COLS <= 32 ? 32 : COLS <= 64 ? 64 : COLS <= 128 ? 128 : COLS <= 256 ? 256 : 512;
  static constexpr int SCHED = 8;  // schedule ring depth
  // readers of a schedule slot: producer, MMA thread, 4 epilogue warps
  static constexpr uint32_t SCHED_READERS = 6;
  // barriers: full[S] empty[S] accf[2] acce[2] schedf[SCHED] schede[SCHED] tmem_ready
  // drain taken
  static constexpr uint32_t NBARS = 2 * STAGES + 4 + 2 * SCHED + 3;
  static constexpr uint32_t MISC_BYTES = 8 * NBARS + 32 * SCHED + 16;
  // carve-out: [operand tiles][scale atoms][barriers, ring, words][epilogue staging]
  static constexpr uint32_t SF_REGION = SUB_SLOTS * OP_BYTES;
  static constexpr uint32_t BAR_REGION = SF_REGION + SUB_SLOTS * SF_BYTES;
  static constexpr uint32_t EPI_REGION = (BAR_REGION + MISC_BYTES + 15) / 16 * 16;
  static constexpr uint32_t SMEM_BYTES = 1024 + EPI_REGION + kEpiStageBytes;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

template <class C>
__global__ void __launch_bounds__(256, 1) fgg_gemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);

  const uint32_t bars = base + C::BAR_REGION;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (C::STAGES + s); };
  auto accf_bar = [&](int b) { return bars + 8u * (2 * C::STAGES + b); };
  auto acce_bar = [&](int b) { return bars + 8u * (2 * C::STAGES + 2 + b); };
  auto schedf_bar = [&](int i) { return bars + 8u * (2 * C::STAGES + 4 + i); };
  auto schede_bar = [&](int i) { return bars + 8u * (2 * C::STAGES + 4 + C::SCHED + i); };
  const uint32_t tmem_ready_bar = bars + 8u * (2 * C::STAGES + 4 + 2 * C::SCHED);
  const uint32_t drain_bar = tmem_ready_bar + 8u;
  const uint32_t taken_bar = tmem_ready_bar + 16u;  // producer took a slot
  uint8_t* const misc = gbase + C::BAR_REGION + 8 * C::NBARS;
  // this warp's epilogue staging (warps 4-7)
  uint32_t* const epi_stage = reinterpret_cast<uint32_t*>(
      gbase + C::EPI_REGION + ((threadIdx.x >> 5) & 3) * (kEpiStageBytes / 4));
  volatile SchedSlot* const ring = reinterpret_cast<volatile SchedSlot*>(misc);
  volatile uint32_t* const tmem_holder =
      reinterpret_cast<volatile uint32_t*>(misc + 32 * C::SCHED);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(misc + 32 * C::SCHED + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // tiles of K-step slot q = stage * KSUB + (K step within the stage)
  auto sW = [&](int q) { return base + q * C::OP_BYTES; };
  auto sX = [&](int q) { return base + q * C::OP_BYTES + C::W_BYTES; };
  auto sSFW = [&](int q) { return base + C::SF_REGION + q * C::SF_BYTES; };
  auto sSFX = [&](int q) { return base + C::SF_REGION + q * C::SF_BYTES + C::SFW_BYTES; };

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
      mbar_init(schede_bar(i), C::SCHED_READERS);
    }
    mbar_init(tmem_ready_bar, 1);
    mbar_init(drain_bar, 1);
    mbar_init(taken_bar, 1);
    *abort_flag = 0;
    if constexpr (!C::MX) {
      // A pack built for a different problem is refused before any load.
      const PackHeader h = *p.pack;
      // reported after griddep_wait: the prepare kernel resets the status word
      if (h.magic != kPackMagic || h.g != p.wg || h.n != p.n || h.k != p.k) *abort_flag = 2;
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

  // Everything above (barriers, TMEM, the weight pack's header) is ready
  // before this launch; the schedule, token descriptors and scale repack come
  // from the prepare kernel just before it on the stream, which this launch
  // may overlap (programmatic dependent launch).
  griddep_wait();
  const bool aborted_early = (*abort_flag != 0);
  if (threadIdx.x == 0 && *abort_flag == 2) atomicCAS(p.status, 0, kStatusBadPack);

  if (warp == 3) {
    // ------------------------------------------------------------ scheduler
    if (lane == 0 && !aborted_early) {
      int slot = 0;
      uint32_t sphase = 0;
      const int num_tiles = p.num_tiles_dev != nullptr ? *p.num_tiles_dev : p.num_tiles;
      for (uint32_t n = 0;; ++n) {
        // Claim tile n only once the producer has taken tile n-1: a CTA holds
        // at most one tile it has not started, so the tail of the tile list
        // spreads over every CTA.  (The producer cannot take tile n before it
        // is published, so the parity below is unambiguous.)
        if (n > 0 && !mbar_wait1(taken_bar, (n - 1) & 1u, abort_flag, p.status,
                                 kStatusTimeoutProducer))
          break;
        const int t = atomicAdd(p.status + 1, 1);
        const uint32_t tile = (t < num_tiles) ? __ldg(p.tiles + t) : kEndTile;
        const SchedSlot s = make_slot<C::MX, C::BN>(p, tile);
        if (!mbar_wait1(schede_bar(slot), sphase ^ 1, abort_flag, p.status,
                        kStatusTimeoutProducer))
          break;
        write_slot(ring, slot, s);
        mbar_arrive(schedf_bar(slot));
        if (++slot == C::SCHED) {
          slot = 0;
          sphase ^= 1;
        }
        if (tile == kEndTile) break;
      }
    }
    __syncwarp();
  } else if (warp == 0) {
    // ------------------------------------------------------------- producer
    // The whole warp runs the loop (operands warp-uniform), one elected lane
    // issues the loads.
    if (!aborted_early) {
      int stage = 0;
      uint32_t phase = 0;
      int slot = 0;
      uint32_t sphase = 0;
      uint32_t arms = 0;
      if (lane == 0) {
        if constexpr (C::MX) prefetch_tensormap(&p.mx_tmap_w);
        if (C::MX || p.x_flat) prefetch_tensormap(&p.tmap_x_flat);
      }
      while (true) {
        if (!mbar_wait(schedf_bar(slot), sphase, abort_flag, p.status, kStatusTimeoutProducer))
          break;
        const uint32_t tile = __shfl_sync(kFullMask, ring[slot].tile, 0);
        const int xtile_index = __shfl_sync(kFullMask, ring[slot].xtile_index, 0);
        const int wgroup = __shfl_sync(kFullMask, ring[slot].wgroup, 0);
        const int row0 = __shfl_sync(kFullMask, ring[slot].row0, 0);
        if (lane == 0) {
          mbar_arrive(schede_bar(slot));
          mbar_arrive(taken_bar);
        }
        if (++slot == C::SCHED) {
          slot = 0;
          sphase ^= 1;
        }
        if (tile == kEndTile) {
          // no new tiles for this CTA: the next kernel on the stream (the next
          // call's prepare kernel) may launch; it waits for this grid's
          // completion before it touches memory
          if (lane == 0) griddep_launch_dependents();
          break;
        }
        const int g = int(tile >> 22);
        const int nti = int((tile >> 11) & 0x7FFu);
        const int xti = int(tile & 0x7FFu);
        // the group and weight group index descriptor arrays: never trust them blindly
        if (g >= p.g || unsigned(wgroup) >= unsigned(p.wg)) {
          if (lane == 0) {
            atomicCAS(p.status, 0, kStatusBadTile);
            *abort_flag = 1;
          }
          break;
        }
        const CUtensorMap* tw;
        const CUtensorMap* tx;
        // first token row of the tile in the map's coordinates
        const int xrow = (C::MX || p.x_flat) ? row0 : xti * C::BN;
        if constexpr (C::MX) {
          tw = &p.mx_tmap_w;
          tx = &p.tmap_x_flat;
        } else {
          tw = p.tmap_w + wgroup;
          tensormap_acquire(tw);  // every lane: the issuing one among them
          if (p.x_flat) {
            tx = &p.tmap_x_flat;
          } else {
            tx = p.tmap_x + g;
            tensormap_acquire(tx);
          }
        }
        const uint8_t* sfx = p.sfx + size_t(xtile_index) * size_t(p.ksteps) * C::SFX_BYTES;
        const uint8_t* sfw =
            p.sfw + (size_t(wgroup) * p.nt + nti) * size_t(p.ksteps) * C::SFW_BYTES;
        bool ok = true;
        for (int ks0 = 0; ks0 < p.ksteps; ks0 += C::KSUB) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.status,
                         kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = full_bar(stage);
          const bool arm = (p.debug_flags & kDebugNoLoads) == 0;
          if (arm && elect_one()) {
            if constexpr (C::KSUB == 1)
              mbar_arrive_expect_tx(fb, C::TX_BYTES);
            else
              mbar_arrive_expect_tx(fb, C::TX_BYTES * uint32_t(min(C::KSUB, p.ksteps - ks0)));
#pragma unroll
            for (int sub = 0; sub < C::KSUB; ++sub) {
              const int ks = ks0 + sub;
              if constexpr (C::KSUB > 1) {
                if (ks >= p.ksteps) break;
              }
              const int q = stage * C::KSUB + sub;
              if constexpr (C::MX)
                tma_load_3d(sW(q), tw, fb, ks * C::K_STEP, nti * 128, g);
              else
                tma_load_2d(sW(q), tw, fb, ks * 128, nti * 128);
              tma_load_2d(sX(q), tx, fb, ks * 128, xrow);
              bulk_g2s(sSFW(q), sfw + size_t(ks) * C::SFW_BYTES, C::SFW_BYTES, fb);
              bulk_g2s(sSFX(q), sfx + size_t(ks) * C::SFX_BYTES, C::SFX_BYTES, fb);
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
      // Every armed stage must land before the CTA may exit (normally already so).
      if (lane == 0) {
        const uint32_t first = arms > uint32_t(C::STAGES) ? arms - C::STAGES : 0u;
        for (uint32_t a = first; a < arms; ++a)
          mbar_wait_one(full_bar(int(a % C::STAGES)), (a / C::STAGES) & 1u, 200000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---------------------------------------------------------- MMA issuer
    // The whole warp runs the loop; the scale uploads, MMAs and commits of a
    // stage issue from one elect.sync region, with every operand (descriptors,
    // TMEM columns) computed outside it and warp-uniform.
    if (!aborted_early) {
      bool ok = mbar_wait(tmem_ready_bar, 0, abort_flag, p.status, kStatusTimeoutMma);
      tc_fence_after();
      const uint32_t tmem = __shfl_sync(kFullMask, *tmem_holder, 0);
      int stage = 0;
      uint32_t phase = 0;
      int slot = 0;
      uint32_t sphase = 0;
      uint32_t lt = 0;
      int sfslot = 0;
      bool issued_any = false;
      while (ok) {
        if (!mbar_wait(schedf_bar(slot), sphase, abort_flag, p.status, kStatusTimeoutMma)) break;
        const uint32_t tile = __shfl_sync(kFullMask, ring[slot].tile, 0);
        const int rows = __shfl_sync(kFullMask, ring[slot].rows, 0);
        if (lane == 0) mbar_arrive(schede_bar(slot));
        if (++slot == C::SCHED) {
          slot = 0;
          sphase ^= 1;
        }
        if (tile == kEndTile) break;
        const int ncols = min(C::BN, (rows + 15) & ~15);
        const uint32_t b = lt & 1u;
        if (!mbar_wait(acce_bar(b), ((lt >> 1) & 1u) ^ 1u, abort_flag, p.status,
                       kStatusTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + b * C::BN;
        const uint32_t idesc =
            C::MX ? 0u : idesc_block_scaled(kFmtNvf4E2M1, kFmtNvf4E2M1, 0, 128, ncols, 0, 0);
        for (int ks0 = 0; ks0 < p.ksteps; ks0 += C::KSUB) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, p.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // scale slots of this stage's MMAs (NVFP4: one per MMA; MX: one per K step)
          constexpr int kSlots = C::KSUB * (C::MX ? 1 : 4);
          uint32_t col[kSlots];
#pragma unroll
          for (int i = 0; i < kSlots; ++i) {
            col[i] = tmem + C::SF_BASE + sfslot * C::SF_SLOT;
            sfslot = (sfslot + 1 == C::NSLOTS) ? 0 : sfslot + 1;
          }
          const bool last = ks0 + C::KSUB >= p.ksteps;
          if (elect_one()) {
#pragma unroll
            for (int sub = 0; sub < C::KSUB; ++sub) {
              const int ks = ks0 + sub;
              if constexpr (C::KSUB > 1) {
                if (ks >= p.ksteps) break;
              }
              const int q = stage * C::KSUB + sub;  // this K step's slot in the stage
              const uint64_t adesc = desc_k_sw128(sW(q));
              const uint64_t bdesc = desc_k_sw128(sX(q));
              if constexpr (C::MX) {
                const uint32_t c0 = col[sub];
                tc_cp_sf(c0, desc_sf_atom(sSFW(q)));
#pragma unroll
                for (int c = 0; c < C::CH; ++c)
                  if (c == 0 || ncols > 128 * c)
                    tc_cp_sf(c0 + 4 + 4 * c, desc_sf_atom(sSFX(q) + c * 512));
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  // K step of 32 one-byte elements = 32 bytes = +2 in the start field;
                  // SF id j picks byte j of every scale column.
                  const uint32_t idj =
                      idesc_block_scaled(kFmtF8E2M1, kFmtF8E4M3, 1, 128, ncols, j, j);
                  tc_mma_mxf8f6f4(d_tmem, adesc + 2u * j, bdesc + 2u * j, idj,
                                  c0 | (uint32_t(j) << 30), (c0 + 4) | (uint32_t(j) << 30),
                                  (ks | j) != 0 ? 1u : 0u);
                }
              } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t c0 = col[sub * 4 + j];
                  tc_cp_sf(c0, desc_sf_atom(sSFW(q) + j * 512));
                  // token scale atom c covers tokens [128 c, 128 c + 128): a tile
                  // of ncols columns reads only the atoms it reaches
#pragma unroll
                  for (int c = 0; c < C::CH; ++c)
                    if (c == 0 || ncols > 128 * c)
                      tc_cp_sf(c0 + 4 + 4 * c, desc_sf_atom(sSFX(q) + (j * C::CH + c) * 512));
                  // K step of 64 fp4 = 32 bytes = +2 in the descriptor's start field.
                  tc_mma_nvf4(d_tmem, adesc + 2u * j, bdesc + 2u * j, idesc, c0, c0 + 4,
                              (ks | j) != 0 ? 1u : 0u);
                }
              }
            }
            tc_commit(empty_bar(stage));
            if (last) tc_commit(accf_bar(b));
          }
          __syncwarp();
          issued_any = true;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ++lt;
      }
      // Drain: every tcgen05 op the warp issued completes before TMEM is freed.
      if (issued_any) {
        if (elect_one()) {
          tc_commit(drain_bar);
          if (!mbar_wait_one(drain_bar, 0, 200000000ull))
            atomicCAS(p.status, 0, kStatusTimeoutDrain);
        }
      }
    }
    __syncwarp();
  } else if (warp >= 4 && !aborted_early) {
    // ------------------------------------------------------------- epilogue
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
      const SchedSlot s = read_slot(ring, slot);
      __syncwarp();
      if (lane == 0) mbar_arrive(schede_bar(slot));
      if (++slot == C::SCHED) {
        slot = 0;
        sphase ^= 1;
      }
      if (s.tile == kEndTile) break;
      const int nti = int((s.tile >> 11) & 0x7FFu);
      const int ncols = min(C::BN, (s.rows + 15) & ~15);
      const uint32_t b = lt & 1u;
      if (!mbar_wait(accf_bar(b), (lt >> 1) & 1u, abort_flag, p.status, kStatusTimeoutEpilogue))
        break;
      tc_fence_after();
      if (p.epi == kEpiSiluMul)
        epilogue_tile_silu_mul(p.out, p.n / 2, nti * 128 + q * 32, size_t(s.row0), s.rows, ncols,
                               s.alpha, tmem + (uint32_t(q * 32) << 16) + b * C::BN);
      else
        epilogue_tile(p.out, p.n, nti * 128 + q * 32, size_t(s.row0), s.rows, ncols, s.alpha,
                      p.row_scale, tmem + (uint32_t(q * 32) << 16) + b * C::BN, epi_stage);
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

// ====================================================================
// CTA-pair engine: cluster (2,1,1), tcgen05 .cta_group::2.
//
// The pair computes a 256 (weight rows) x 224 (tokens) tile: each CTA loads
// its own 128 weight rows and HALF of the token rows, so the token tile
// crosses L2 -> SM once per pair instead of once per CTA.  The leader (rank 0)
// runs the scheduler (it publishes every slot into both CTAs' rings), arms one
// full barrier per stage for both CTAs' bytes (every load of the pair books
// its completion there: .cta_group::2 TMA), and issues the scale-factor
// uploads and MMAs.  Commits arrive in both CTAs (empty stages, accumulator
// ready); each CTA's epilogue drains its own TMEM (its 128 output columns) and
// tells the leader's acc-empty barrier when it is done.
// Scale factors: each CTA holds the atoms of its own weight rows and the atoms
// of all 224 tokens; the leader's tcgen05.cp.cta_group::2 copies each CTA's
// atoms into that CTA's TMEM.
// Waits acquire at CTA scope (TMA / tcgen05 completions), except on the
// schedule ring, whose slots the leader writes into the follower's shared
// memory: those waits acquire at cluster scope.
// ====================================================================
template <bool MX_, int STAGES_, int KSUB_ = 1>
struct PairCfg {
  static constexpr bool MX = MX_;
  static constexpr int BN = 224;   // tokens per pair tile = MMA N
  static constexpr int BNH = 112;  // token rows one CTA loads
  static constexpr int STAGES = STAGES_;
  // K steps per pipeline stage: one barrier wait and one commit on the MMA
  // thread cover KSUB K steps
  static constexpr int KSUB = KSUB_;
  static_assert(KSUB == 1 || KSUB == 2, "one or two K steps per stage");
  static constexpr int CH = 2;     // 128-row token SF atoms per tile
  static constexpr int K_STEP = MX ? 128 : 256;
  static constexpr uint32_t W_BYTES = 128 * 128;
  static constexpr uint32_t W_TX = MX ? 64 * 128 : 128 * 128;
  static constexpr uint32_t X_BYTES = BNH * 128;
  // Weight scales of a K step (this CTA's 128 rows).  MX: one atom for the 4
  // MMAs.  NVFP4: one atom per MMA.
  static constexpr uint32_t SFW_BYTES = MX ? 512 : 4 * 512;
  // token scales of all 224 tokens: two atoms per MMA (NVFP4) or per K step (MX)
  static constexpr uint32_t SFX_BYTES = MX ? 2 * 512 : 4 * 2 * 512;
  // SF atoms travel as 2-D uint64 boxes {ROW_U64, BOX_ROWS}
  static constexpr uint32_t SFW_ROW_U64 = SFW_BYTES / 8 > 256 ? 256 : SFW_BYTES / 8;
  static constexpr uint32_t SFW_BOX_ROWS = SFW_BYTES / (8 * SFW_ROW_U64);
  static constexpr uint32_t SFX_ROW_U64 = SFX_BYTES / 8 > 256 ? 256 : SFX_BYTES / 8;
  static constexpr uint32_t SFX_BOX_ROWS = SFX_BYTES / (8 * SFX_ROW_U64);
  static constexpr uint32_t TX_CTA = W_TX + X_BYTES + SFW_BYTES + SFX_BYTES;
  // operand tiles and scale atoms of a K step in separate regions (see EngineCfg)
  static constexpr uint32_t OP_BYTES = W_BYTES + X_BYTES;
  static constexpr uint32_t SF_BYTES = SFW_BYTES + SFX_BYTES;
  static constexpr uint32_t SUB_SLOTS = STAGES_ * KSUB;
  static_assert(OP_BYTES % 1024 == 0, "operand tiles must stay 1024 B aligned");
  static_assert(SF_BYTES % 128 == 0, "scale atoms must stay 128 B aligned");
  static constexpr int SF_BASE = 2 * BN;          // 448
  // [weights 4 | tokens 8]: per MMA (NVFP4) or per K step (MX)
  static constexpr int SF_SLOT = 12;
  static constexpr int NSLOTS = (512 - SF_BASE) / SF_SLOT;
  static_assert(NSLOTS >= 2, "not enough TMEM for the scale ring");
  static_assert(SF_BASE + NSLOTS * SF_SLOT <= 512, "TMEM columns exceeded");
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr int SCHED = 8;
  // readers of a slot: leader producer, MMA thread, 4 epilogue warps; follower
  // producer and 4 epilogue warps
  static constexpr uint32_t SCHED_READERS = 11;
  static constexpr uint32_t NBARS = 2 * STAGES + 4 + 2 * SCHED + 3;
  static constexpr uint32_t MISC_BYTES = 8 * NBARS + 32 * SCHED + 16;
  static constexpr uint32_t SF_REGION = SUB_SLOTS * OP_BYTES;
  static constexpr uint32_t BAR_REGION = SF_REGION + SUB_SLOTS * SF_BYTES;
  static constexpr uint32_t EPI_REGION = (BAR_REGION + MISC_BYTES + 15) / 16 * 16;
  static constexpr uint32_t SMEM_BYTES = 1024 + EPI_REGION + kEpiStageBytes;
  static_assert(SMEM_BYTES <= 232448, "shared memory budget exceeded");
};

template <class C>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 1)
    fgg_gemm_pair_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* const gbase = smem_raw + (base - raw);

  const uint32_t bars = base + C::BAR_REGION;
  auto full_bar = [&](int s) { return bars + 8u * s; };
  auto empty_bar = [&](int s) { return bars + 8u * (C::STAGES + s); };
  auto accf_bar = [&](int b) { return bars + 8u * (2 * C::STAGES + b); };
  auto acce_bar = [&](int b) { return bars + 8u * (2 * C::STAGES + 2 + b); };
  auto schedf_bar = [&](int i) { return bars + 8u * (2 * C::STAGES + 4 + i); };
  auto schede_bar = [&](int i) { return bars + 8u * (2 * C::STAGES + 4 + C::SCHED + i); };
  const uint32_t tmem_ready_bar = bars + 8u * (2 * C::STAGES + 4 + 2 * C::SCHED);
  const uint32_t drain_bar = tmem_ready_bar + 8u;
  const uint32_t taken_bar = tmem_ready_bar + 16u;  // producer took a slot
  uint8_t* const misc = gbase + C::BAR_REGION + 8 * C::NBARS;
  // this warp's epilogue staging (warps 4-7)
  uint32_t* const epi_stage = reinterpret_cast<uint32_t*>(
      gbase + C::EPI_REGION + ((threadIdx.x >> 5) & 3) * (kEpiStageBytes / 4));
  volatile SchedSlot* const ring = reinterpret_cast<volatile SchedSlot*>(misc);
  volatile uint32_t* const tmem_holder =
      reinterpret_cast<volatile uint32_t*>(misc + 32 * C::SCHED);
  volatile int* const abort_flag = reinterpret_cast<volatile int*>(misc + 32 * C::SCHED + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = (rank == 0);
  const uint32_t peer = rank ^ 1u;

  // tiles of K-step slot q = stage * KSUB + (K step within the stage)
  auto sW = [&](int q) { return base + q * C::OP_BYTES; };
  auto sX = [&](int q) { return base + q * C::OP_BYTES + C::W_BYTES; };
  auto sSFW = [&](int q) { return base + C::SF_REGION + q * C::SF_BYTES; };
  auto sSFX = [&](int q) { return base + C::SF_REGION + q * C::SF_BYTES + C::SFW_BYTES; };
  // MMA N of a tile: a multiple of 32 so that each CTA holds a multiple of 16 rows
  auto tile_ncols = [&](int rows) -> int { return min(C::BN, (rows + 31) & ~31); };

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(accf_bar(b), 1);
      mbar_init(acce_bar(b), 8);  // 4 epilogue warps in each CTA (leader's barrier)
    }
    for (int i = 0; i < C::SCHED; ++i) {
      mbar_init(schedf_bar(i), 1);
      mbar_init(schede_bar(i), C::SCHED_READERS);  // used on the leader
    }
    mbar_init(tmem_ready_bar, 1);
    mbar_init(drain_bar, 1);
    mbar_init(taken_bar, 1);
    *abort_flag = 0;
    if constexpr (!C::MX) {
      const PackHeader h = *p.pack;
      // reported after griddep_wait: the prepare kernel resets the status word
      if (h.magic != kPackMagic || h.g != p.wg || h.n != p.n || h.k != p.k) *abort_flag = 2;
    }
    fence_mbar_init();
  }
  // barrier inits visible to the peer before any of its loads or arrivals
  cluster_sync();

  if (warp == 2) {
    tmem_alloc_pair(smem_u32(const_cast<uint32_t*>(tmem_holder)), C::TMEM_COLS);
    tmem_relinquish_pair();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(tmem_ready_bar);
  }

  // Everything above (barriers, TMEM, the weight pack's header) is ready
  // before this launch; the schedule, token descriptors and scale repack come
  // from the prepare kernel just before it on the stream, which this launch
  // may overlap (programmatic dependent launch).
  griddep_wait();
  const bool aborted_early = (*abort_flag != 0);
  if (threadIdx.x == 0 && *abort_flag == 2) atomicCAS(p.status, 0, kStatusBadPack);
  const uint32_t leader_schede0 = mapa_shared(schede_bar(0), 0);
  const uint32_t leader_acce0 = mapa_shared(acce_bar(0), 0);
  const uint32_t leader_full0 = mapa_shared(full_bar(0), 0);

  // release a slot this thread has read: the leader's ring barrier counts the
  // readers of both CTAs
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
        // one unstarted tile per pair at most (see the single-CTA kernel)
        if (n > 0 && !mbar_wait1(taken_bar, (n - 1) & 1u, abort_flag, p.status,
                                 kStatusTimeoutProducer))
          break;
        const int t = atomicAdd(p.status + 1, 1);
        const uint32_t tile = (t < num_tiles) ? __ldg(p.tiles + t) : kEndTile;
        const SchedSlot s = make_slot<C::MX, C::BN>(p, tile);
        if (!mbar_wait1<true>(schede_bar(slot), sphase ^ 1, abort_flag, p.status,
                              kStatusTimeoutProducer))
          break;
        write_slot(ring, slot, s);
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
    // The whole warp runs the loop (operands warp-uniform), one elected lane
    // issues the loads.
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
        const int rows = __shfl_sync(kFullMask, ring[slot].rows, 0);
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
          if (lane == 0) griddep_launch_dependents();  // as in the single-CTA kernel
          break;
        }
        const int g = int(tile >> 22);
        const int nti = int((tile >> 11) & 0x7FFu);
        const int xti = int(tile & 0x7FFu);
        // the group and weight group index descriptor arrays: never trust them blindly
        if (g >= p.g || unsigned(wgroup) >= unsigned(p.wg)) {
          if (lane == 0) {
            atomicCAS(p.status, 0, kStatusBadTile);
            *abort_flag = 1;
          }
          break;
        }
        const int half = tile_ncols(rows) >> 1;
        const CUtensorMap* tw;
        const CUtensorMap* tx;
        // bytes both CTAs' loads of one K step deliver to the leader's barrier
        uint32_t tx_step = 2u * C::TX_CTA;
        if constexpr (C::MX) {
          tw = &p.mx_tmap_w;
          tx = &p.tmap_x_flat;
        } else {
          tw = p.tmap_w + wgroup;
          tensormap_acquire(tw);  // every lane: the issuing one among them
          if (p.x_flat) {
            tx = &p.tmap_x_flat;
            // a narrow tile (half a multiple of 16 below BNH) loads its rows only
            if (p.x_small && half >= 16 && half < C::BNH) {
              tx = &p.tmap_x_small[half / 16 - 1];
              tx_step = 2u * (C::TX_CTA - C::X_BYTES + uint32_t(half) * 128u);
            }
          } else {
            tx = p.tmap_x + g;
            tensormap_acquire(tx);
          }
        }
        const int wrow = nti * 256 + int(rank) * 128;
        // this CTA's first token row in the map's coordinates
        const int xrow = ((C::MX || p.x_flat) ? row0 : xti * C::BN) + int(rank) * half;
        // this CTA's weight scale atoms of the tile: one row of SFW_BYTES per K step
        const int sfw_y =
            ((wgroup * p.nt128 + 2 * nti + int(rank)) * p.ksteps) * int(C::SFW_BOX_ROWS);
        const int sfx_y = (xtile_index * p.ksteps) * int(C::SFX_BOX_ROWS);
        bool ok = true;
        for (int ks0 = 0; ks0 < p.ksteps; ks0 += C::KSUB) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, abort_flag, p.status,
                         kStatusTimeoutProducer)) {
            ok = false;
            break;
          }
          const uint32_t fb = leader_full0 + 8u * stage;
          const bool arm = (p.debug_flags & kDebugNoLoads) == 0;
          if (arm && elect_one()) {
            if (leader) {
              if constexpr (C::KSUB == 1)
                mbar_arrive_expect_tx(full_bar(stage), tx_step);
              else
                mbar_arrive_expect_tx(full_bar(stage),
                                      tx_step * uint32_t(min(C::KSUB, p.ksteps - ks0)));
            }
#pragma unroll
            for (int sub = 0; sub < C::KSUB; ++sub) {
              const int ks = ks0 + sub;
              if constexpr (C::KSUB > 1) {
                if (ks >= p.ksteps) break;
              }
              const int q = stage * C::KSUB + sub;
              if constexpr (C::MX)
                tma_load_3d_pair(sW(q), tw, fb, ks * C::K_STEP, wrow, g);
              else
                tma_load_2d_pair(sW(q), tw, fb, ks * 128, wrow);
              tma_load_2d_pair(sX(q), tx, fb, ks * 128, xrow);
              tma_load_2d_pair(sSFW(q), &p.sfw_map, fb, 0, sfw_y + ks * int(C::SFW_BOX_ROWS));
              tma_load_2d_pair(sSFX(q), &p.sfx_map, fb, 0, sfx_y + ks * int(C::SFX_BOX_ROWS));
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
      // the leader's full barriers cover both CTAs' bytes: drain them before exit
      if (leader && lane == 0) {
        const uint32_t first = arms > uint32_t(C::STAGES) ? arms - C::STAGES : 0u;
        for (uint32_t a = first; a < arms; ++a)
          mbar_wait_one(full_bar(int(a % C::STAGES)), (a / C::STAGES) & 1u, 200000000ull);
      }
    }
    __syncwarp();
  } else if (warp == 1 && leader) {
    // ------------------------------------------------------- MMA issuer
    // The whole warp runs the loop; one elect.sync region per stage issues its
    // scale uploads, MMAs and commits with warp-uniform operands.
    if (!aborted_early) {
      bool ok = mbar_wait(tmem_ready_bar, 0, abort_flag, p.status, kStatusTimeoutMma);
      tc_fence_after();
      const uint32_t tmem = __shfl_sync(kFullMask, *tmem_holder, 0);
      int stage = 0;
      uint32_t phase = 0;
      int slot = 0;
      uint32_t sphase = 0;
      uint32_t lt = 0;
      int sfslot = 0;
      bool issued_any = false;
      while (ok) {
        if (!mbar_wait<true>(schedf_bar(slot), sphase, abort_flag, p.status, kStatusTimeoutMma))
          break;
        const uint32_t tile = __shfl_sync(kFullMask, ring[slot].tile, 0);
        const int rows = __shfl_sync(kFullMask, ring[slot].rows, 0);
        if (lane == 0) mbar_arrive(schede_bar(slot));
        if (++slot == C::SCHED) {
          slot = 0;
          sphase ^= 1;
        }
        if (tile == kEndTile) break;
        const int ncols = tile_ncols(rows);
        const uint32_t b = lt & 1u;
        if (!mbar_wait(acce_bar(b), ((lt >> 1) & 1u) ^ 1u, abort_flag, p.status,
                       kStatusTimeoutMma))
          break;
        tc_fence_after();
        const uint32_t d_tmem = tmem + b * C::BN;
        const uint32_t idesc =
            C::MX ? 0u : idesc_block_scaled(kFmtNvf4E2M1, kFmtNvf4E2M1, 0, 256, ncols, 0, 0);
        for (int ks0 = 0; ks0 < p.ksteps; ks0 += C::KSUB) {
          if (!mbar_wait(full_bar(stage), phase, abort_flag, p.status, kStatusTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // scale slots of this stage's MMAs (NVFP4: one per MMA; MX: one per K step)
          constexpr int kSlots = C::KSUB * (C::MX ? 1 : 4);
          uint32_t col[kSlots];
#pragma unroll
          for (int i = 0; i < kSlots; ++i) {
            col[i] = tmem + C::SF_BASE + sfslot * C::SF_SLOT;
            sfslot = (sfslot + 1 == C::NSLOTS) ? 0 : sfslot + 1;
          }
          const bool last = ks0 + C::KSUB >= p.ksteps;
          if (elect_one()) {
#pragma unroll
            for (int sub = 0; sub < C::KSUB; ++sub) {
              const int ks = ks0 + sub;
              if constexpr (C::KSUB > 1) {
                if (ks >= p.ksteps) break;
              }
              const int q = stage * C::KSUB + sub;  // this K step's slot in the stage
              const uint64_t adesc = desc_k_sw128(sW(q));
              const uint64_t bdesc = desc_k_sw128(sX(q));
              if constexpr (C::MX) {
                const uint32_t c0 = col[sub];
                tc_cp_sf_pair(c0, desc_sf_atom(sSFW(q)));
                tc_cp_sf_pair(c0 + 4, desc_sf_atom(sSFX(q)));
                if (ncols > 128) tc_cp_sf_pair(c0 + 8, desc_sf_atom(sSFX(q) + 512));
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t idj =
                      idesc_block_scaled(kFmtF8E2M1, kFmtF8E4M3, 1, 256, ncols, j, j);
                  tc_mma_mxf8f6f4_pair(d_tmem, adesc + 2u * j, bdesc + 2u * j, idj,
                                       c0 | (uint32_t(j) << 30), (c0 + 4) | (uint32_t(j) << 30),
                                       (ks | j) != 0 ? 1u : 0u);
                }
              } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint32_t c0 = col[sub * 4 + j];
                  tc_cp_sf_pair(c0, desc_sf_atom(sSFW(q) + j * 512));
                  tc_cp_sf_pair(c0 + 4, desc_sf_atom(sSFX(q) + (2 * j) * 512));
                  // tokens 128..223: only a tile wider than 128 columns reads them
                  if (ncols > 128)
                    tc_cp_sf_pair(c0 + 8, desc_sf_atom(sSFX(q) + (2 * j + 1) * 512));
                  tc_mma_nvf4_pair(d_tmem, adesc + 2u * j, bdesc + 2u * j, idesc, c0, c0 + 4,
                                   (ks | j) != 0 ? 1u : 0u);
                }
              }
            }
            tc_commit_pair(empty_bar(stage), 0x3);
            if (last) tc_commit_pair(accf_bar(b), 0x3);
          }
          __syncwarp();
          issued_any = true;
          if (++stage == C::STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        ++lt;
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
    const int q = warp & 3;
    bool ok = mbar_wait(tmem_ready_bar, 0, abort_flag, p.status, kStatusTimeoutEpilogue);
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    int slot = 0;
    uint32_t sphase = 0;
    uint32_t lt = 0;
    while (ok) {
      if (!mbar_wait<true>(schedf_bar(slot), sphase, abort_flag, p.status,
                           kStatusTimeoutEpilogue))
        break;
      const SchedSlot s = read_slot(ring, slot);
      __syncwarp();
      if (lane == 0) release_slot(slot);
      if (++slot == C::SCHED) {
        slot = 0;
        sphase ^= 1;
      }
      if (s.tile == kEndTile) break;
      const int nti = int((s.tile >> 11) & 0x7FFu);
      const int ncols = tile_ncols(s.rows);
      const uint32_t b = lt & 1u;
      if (!mbar_wait(accf_bar(b), (lt >> 1) & 1u, abort_flag, p.status, kStatusTimeoutEpilogue))
        break;
      tc_fence_after();
      if (p.epi == kEpiSiluMul)
        epilogue_tile_silu_mul(p.out, p.n / 2, nti * 256 + int(rank) * 128 + q * 32,
                               size_t(s.row0), s.rows, ncols, s.alpha,
                               tmem + (uint32_t(q * 32) << 16) + b * C::BN);
      else
        epilogue_tile(p.out, p.n, nti * 256 + int(rank) * 128 + q * 32, size_t(s.row0), s.rows,
                      ncols, s.alpha, p.row_scale, tmem + (uint32_t(q * 32) << 16) + b * C::BN,
                      epi_stage);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (leader)
          mbar_arrive(acce_bar(b));
        else
          mbar_arrive_remote(leader_acce0 + 8u * b);
      }
      ++lt;
    }
  }

  __syncthreads();
  // the leader's MMAs write the follower's TMEM and read its shared memory:
  // neither CTA frees anything before both are done
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

// Launch a kernel as a programmatic dependent of the preceding kernel on the
// stream: it may start while that kernel finishes (the GEMM behind the
// prepare kernel, the next call's prepare kernel behind a GEMM's last tiles),
// and waits for its results at griddep_wait().  Host only.
template <class Kernel, class Params>
cudaError_t launch_dependent(Kernel kernel, int grid, uint32_t smem, cudaStream_t s,
                             const Params& gp) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, gp);
}

// Raise the kernel's dynamic shared memory limit (once per context), then launch
// one CTA pair per two SMs, or one per tile when there are fewer tiles.  Host only.
template <class C>
cudaError_t launch_pair(const GemmParams& gp, int sm_count, cudaStream_t s) {
  if (ensure_max_dynamic_smem(reinterpret_cast<const void*>(fgg_gemm_pair_kernel<C>),
                              int(C::SMEM_BYTES)) != FGG_OK)
    return cudaErrorInvalidValue;
  const int pairs_avail = sm_count / 2;
  const int pairs = gp.num_tiles < pairs_avail ? (gp.num_tiles > 0 ? gp.num_tiles : 1) : pairs_avail;
  return launch_dependent(fgg_gemm_pair_kernel<C>, 2 * pairs, C::SMEM_BYTES, s, gp);
}

// Raise the kernel's dynamic shared memory limit (once per context), then launch
// one CTA per SM, or one per tile when there are fewer tiles.  Host only.
template <class C>
cudaError_t launch_engine(const GemmParams& gp, int sm_count, cudaStream_t s) {
  if (ensure_max_dynamic_smem(reinterpret_cast<const void*>(fgg_gemm_kernel<C>),
                              int(C::SMEM_BYTES)) != FGG_OK)
    return cudaErrorInvalidValue;
  const int grid = gp.num_tiles < sm_count ? (gp.num_tiles > 0 ? gp.num_tiles : 1) : sm_count;
  return launch_dependent(fgg_gemm_kernel<C>, grid, C::SMEM_BYTES, s, gp);
}

}  // namespace fgg
