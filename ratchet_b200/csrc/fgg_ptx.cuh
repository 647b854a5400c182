// fgg_ptx.cuh - thin inline-PTX layer for sm_100a: mbarriers, TMA, bulk
// copies, tensormap edits, and the tcgen05 family (TMEM alloc, block-scaled
// MMA, SF upload, TMEM readback).  Every wait is bounded: it gives up after
// kWaitLimitNs of %globaltimer time or as soon as the CTA's abort word is set,
// records a status code in global memory and returns false, so a broken
// pipeline ends the kernel instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace fgg {

constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s per wait

// status word codes (workspace word 0)
constexpr int kStatusOk = 0;
constexpr int kStatusTimeoutProducer = 0x101;
constexpr int kStatusTimeoutMma = 0x102;
constexpr int kStatusTimeoutEpilogue = 0x103;
constexpr int kStatusTimeoutDrain = 0x104;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

constexpr unsigned kFullMask = 0xffffffffu;

// One lane of a converged warp (elect.sync over the full mask).  The producer
// and MMA roles run their loops on the whole warp, so every operand of a TMA or
// tcgen05 instruction is warp-uniform, and issue from the elected lane.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, e;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
// Upper bound (ns) a waiting thread stays suspended inside one try_wait: the
// hardware wakes it as soon as the phase completes, so waiting warps sleep
// instead of spinning and stealing issue slots from the MMA thread.
constexpr uint32_t kSuspendHintNs = 1000000u;

// kCluster: acquire at cluster scope, for barriers the peer CTA of a pair
// arrives on after writing this CTA's shared memory.
template <bool kCluster = false>
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  if constexpr (kCluster) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
        : "memory");
  }
  return ok != 0;
}

// Bounded wait executed by every lane of a warp; the outcome is warp-uniform.
// `abort_flag` is a CTA-wide shared word: once any role gives up, the others
// stop waiting immediately.  `status` is the kernel's global status word.
template <bool kCluster = false>
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity,
                                          volatile int* abort_flag, int* status,
                                          int code) {
  bool ok = mbar_try_wait<kCluster>(bar, parity);
  if (!__all_sync(0xffffffffu, ok)) {
    const uint64_t t0 = globaltimer();
    while (true) {
      if (!ok) ok = mbar_try_wait<kCluster>(bar, parity);
      if (__all_sync(0xffffffffu, ok)) break;
      const bool give_up = (*abort_flag != 0) || (globaltimer() - t0 > kWaitLimitNs);
      if (__any_sync(0xffffffffu, give_up)) {
        if ((threadIdx.x & 31) == 0) {
          atomicCAS(status, 0, code);
          *abort_flag = 1;
        }
        __syncwarp();
        return false;
      }
    }
  }
  return true;
}

// Bounded wait executed by ONE thread (the tile scheduler, which runs on a
// single lane).  Checks the clock and the abort word after every poll.
template <bool kCluster = false>
__device__ __forceinline__ bool mbar_wait1(uint32_t bar, uint32_t parity,
                                           volatile int* abort_flag, int* status, int code) {
  if (mbar_try_wait<kCluster>(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait<kCluster>(bar, parity)) return true;
    {
      if (*abort_flag != 0 || globaltimer() - t0 > kWaitLimitNs) {
        atomicCAS(status, 0, code);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Same, for a single thread (teardown drains).
__device__ __forceinline__ bool mbar_wait_one(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer() - t0 > limit_ns) return false;
  }
  return true;
}

// ------------------------------------------------------------ TMA / bulk
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// Plain (untiled) bulk copy global -> shared; 16-byte aligned, size % 16 == 0.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Consumer side of a descriptor written by another kernel through the generic proxy.
__device__ __forceinline__ void tensormap_acquire(const CUtensorMap* map) {
  asm volatile("fence.proxy.tensormap::generic.acquire.gpu [%0], 128;" ::"l"(
                   reinterpret_cast<uint64_t>(map))
               : "memory");
}

// ------------------------------------------------------- tensormap edits
__device__ __forceinline__ void tmap_replace_address(uint32_t smem_map, uint64_t addr) {
  asm volatile("tensormap.replace.tile.global_address.shared::cta.b1024.b64 [%0], %1;" ::"r"(
                   smem_map),
               "l"(addr)
               : "memory");
}
__device__ __forceinline__ void tmap_replace_dim1(uint32_t smem_map, int32_t extent) {
  asm volatile("tensormap.replace.tile.global_dim.shared::cta.b1024.b32 [%0], 1, %1;" ::"r"(
                   smem_map),
               "r"(extent)
               : "memory");
}
// Warp-collective copy of an edited descriptor from shared to global memory,
// with the release fence that publishes it to the tensormap proxy.
__device__ __forceinline__ void tmap_publish(CUtensorMap* gdst, uint32_t smem_map) {
  asm volatile(
      "tensormap.cp_fenceproxy.global.shared::cta.tensormap::generic.release.gpu.sync.aligned"
      " [%0], [%1], 128;" ::"l"(reinterpret_cast<uint64_t>(gdst)),
      "r"(smem_map)
      : "memory");
}

// ------------------------------------------- programmatic dependent launch
// Primary side: this block no longer holds back the launch of the next grid
// on the stream (which must still wait for this grid's results, below).
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Dependent side: wait until the preceding grid on the stream has completed
// and its memory is visible.  Returns at once when no such dependency exists.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// --------------------------------------------------------------- clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
// Arrive on an mbarrier of another CTA of the cluster (release at cluster scope
// orders this thread's earlier shared-memory writes, remote ones included).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar)
               : "memory");
}
__device__ __forceinline__ void st_shared_remote_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
// 2-D TMA load by one CTA of a pair whose completion is booked on an mbarrier
// that may live in the peer CTA (the leader's).  The box lands only in the
// issuing CTA's own shared memory.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t cluster_bar, int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t cluster_bar, int32_t x, int32_t y,
                                                 int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(cluster_bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// --------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t holder_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   holder_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrive on `bar` once every tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
// 32 lanes x 128 bit from shared memory, replicated into the four 32-lane
// quadrants of TMEM: the scale-factor upload shape the block-scaled MMA reads.
__device__ __forceinline__ void tc_cp_sf(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T with per-16-element E4M3 block scales read from TMEM.
__device__ __forceinline__ void tc_mma_nvf4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X"
      " [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}
// MXF8F6F4 family with one UE8M0 scale per 32 K elements (the reference format).
__device__ __forceinline__ void tc_mma_mxf8f6f4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t sfa_tmem,
                                                uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale"
      " [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}
// ---- CTA-pair (cta_group::2) forms: issued by the pair's leader (alloc and
// dealloc by the same warp in both CTAs); operands are read from both CTAs'
// shared memory at the same offsets and results land in both CTAs' TMEM.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t holder_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   holder_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
// Arrive on the barrier at the same offset in every CTA named by `cta_mask`
// once this thread's earlier tcgen05 ops complete.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}
__device__ __forceinline__ void tc_cp_sf_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc)
               : "memory");
}
__device__ __forceinline__ void tc_mma_nvf4_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t sfa_tmem,
                                                 uint32_t sfb_tmem, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X"
      " [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_mma_mxf8f6f4_pair(uint32_t d_tmem, uint64_t adesc,
                                                     uint64_t bdesc, uint32_t idesc,
                                                     uint32_t sfa_tmem, uint32_t sfb_tmem,
                                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale"
      " [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(sfa_tmem), "r"(sfb_tmem), "r"(accumulate)
      : "memory");
}

// Each thread reads 16 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ----------------------------------------------------------- descriptors
// Shared-memory matrix descriptor (sm_100 format, version bit 46 set).
//   [0,14) start>>4  [16,30) LBO>>4  [32,46) SBO>>4  [46,48) version=1
//   [49,52) base offset (0: tiles are 1024 B aligned)  [61,64) layout type
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t layout) {
  const uint64_t lo = ((saddr >> 4) & 0x3FFFu) | (((lbo >> 4) & 0x3FFFu) << 16);
  const uint64_t hi = ((sbo >> 4) & 0x3FFFu) | (1u << 14) | (layout << 29);
  return lo | (hi << 32);
}
constexpr uint32_t kLayoutSwizzle128 = 2;
constexpr uint32_t kLayoutNone = 0;

// K-major operand tile written by TMA with 128-byte swizzle: 8-row groups of
// 128-byte rows, 1024 B apart.  Stepping K inside the 128 B row adds to the
// start address (the hardware swizzles from the address bits).
__device__ __forceinline__ uint64_t desc_k_sw128(uint32_t saddr) {
  return smem_desc(saddr, 16, 1024, kLayoutSwizzle128);
}
// Scale-factor atom (512 B = 32 rows x 16 B, core matrices of 8 x 16 B).
__device__ __forceinline__ uint64_t desc_sf_atom(uint32_t saddr) {
  return smem_desc(saddr, 128, 128, kLayoutNone);
}

// Instruction descriptor, block-scaled kinds (bit fields from the PTX ISA
// "Instruction descriptor" table for .kind::mxf8f6f4 / .kind::mxf4nvf4):
//   [4,6) B scale id  [7,10) A format  [10,13) B format  [15] A MN-major
//   [16] B MN-major  [17,23) N>>3  [23] scale format (0 E4M3, 1 E8M0)
//   [24,29) M>>4  [29,31) A scale id  [31] K size
__host__ __device__ constexpr uint32_t idesc_block_scaled(uint32_t afmt, uint32_t bfmt,
                                                          uint32_t scale_ue8m0, int m, int n,
                                                          uint32_t a_sf_id, uint32_t b_sf_id) {
  return (b_sf_id << 4) | (afmt << 7) | (bfmt << 10) | (uint32_t(n >> 3) << 17) |
         (scale_ue8m0 << 23) | (uint32_t(m >> 4) << 24) | (a_sf_id << 29);
}
constexpr uint32_t kFmtNvf4E2M1 = 1;   // .kind::mxf4nvf4 operand format E2M1
constexpr uint32_t kFmtF8E4M3 = 0;     // .kind::mxf8f6f4 E4M3
constexpr uint32_t kFmtF8E2M1 = 5;     // .kind::mxf8f6f4 E2M1 (one element per byte in smem)

}  // namespace fgg
