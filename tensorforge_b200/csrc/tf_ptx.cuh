// tf_ptx.cuh -- inline-PTX wrappers for sm_100a: mbarriers with bounded waits, TMA
// tile loads, tcgen05 tensor-memory allocation, MMA, commit and loads.
//
// Every wait in this library is bounded: a waiter polls `mbarrier.try_wait` and reads
// %globaltimer every few polls; past the limit it raises the CTA's abort flag, writes
// TFORGE_ERR_TIMEOUT into the device status word and returns false, so the kernel can
// drain and exit instead of hanging the GPU.
#pragma once
#include <cstdint>

namespace tf {

constexpr uint32_t kStatusTimeout = 6;  // == TFORGE_ERR_TIMEOUT

// Grouped raster of a tiles_m x tiles_n tile grid: tile number `pid` walks `group` tile rows
// at a time, column by column, so the tiles in flight share a few A row panels and B column
// panels in L2.
__device__ __forceinline__ void raster_tile(int pid, int tiles_m, int tiles_n, int group, int &tile_m,
                                            int &tile_n) {
  const int per_group = group * tiles_n, g = pid / per_group;
  const int first_m = g * group;
  const int group_m = tiles_m - first_m < group ? tiles_m - first_m : group;
  tile_m = first_m + (pid - g * per_group) % group_m;
  tile_n = (pid - g * per_group) / group_m;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier -------------------------------------------------------------------
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
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Per-CTA control block for bounded waits (lives in shared memory).
struct WaitCtl {
  volatile uint32_t *abort;  // shared flag: nonzero once any waiter gave up
  uint32_t *status;          // device status word (global)
  uint64_t limit_ns;
};

static __device__ __noinline__ void raise_timeout(const WaitCtl &c) {
  *c.abort = 1u;
  atomicCAS(c.status, 0u, kStatusTimeout);
}

// Returns true when the phase with `parity` completed, false if this CTA aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const WaitCtl &c) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*c.abort) return false;
    if (globaltimer() - t0 > c.limit_ns) {
      raise_timeout(c);
      return false;
    }
  }
}

// Bounded wait used on drain paths after an abort: never raises, just gives up.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > limit_ns) return false;
  }
}

// ---- TMA ----------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void *tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
// 2-D tiled load global -> shared, completion counted on `bar` (bytes).  No multicast.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void *tmap, int32_t c0, int32_t c1,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

// CTA-pair form: the tile lands in this CTA's shared memory at `dst`; completion is
// counted on the mbarrier at cluster address `bar_cluster`, which may be in the peer CTA
// of the pair (the leader's barrier collects both CTAs' bytes).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void *tmap, int32_t c0, int32_t c1,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}

// 4-D tiled loads (the k-group-major B tile, b_mn_desc); same completion as the 2-D forms.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void *tmap, int32_t c0, int32_t c1, int32_t c2,
                                            int32_t c3, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d_pair(uint32_t dst, const void *tmap, int32_t c0, int32_t c1, int32_t c2,
                                                 int32_t c3, uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar_cluster)
      : "memory");
}

// 2-D tiled store shared -> global (bulk-group completion); TMA clips rows and columns
// outside the tensor.  Coordinates must be non-negative.
__device__ __forceinline__ void tma_store_2d(const void *tmap, uint32_t src, int32_t c0, int32_t c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          reinterpret_cast<uint64_t>(tmap)),
      "r"(c0), "r"(c1), "r"(src)
      : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until every committed bulk store of this thread has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// The same, except that the most recently committed group may still be reading.
__device__ __forceinline__ void bulk_wait_group_read1() {
  asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
}
// Named barrier over `count` threads (ids 1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_barrier(uint32_t id, uint32_t count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Programmatic dependent launch.  grid_dependency_wait: block until the grid this launch
// depends on has completed and its memory writes are visible (immediately, when the launch
// had no programmatic dependency).  grid_launch_dependents: let the grids that depend on this
// one start launching (their CTAs can set up while this grid finishes).
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Generic-proxy writes to shared memory -> visible to the async proxy (tcgen05.mma).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- tcgen05 ------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
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

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32 or kind::f16 (bf16 inputs).
template <bool kTF32>
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  if constexpr (kTF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}

// Arrive on `bar` once every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane (base lane + t).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// tmem_ld_wait, then an empty asm that reads and rewrites the 32 destination registers: it is
// ordered after the wait (both volatile), so no use of r can be scheduled above the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  tmem_ld_wait();
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),
                 "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),
                 "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),
                 "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),
                 "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31]));
}

// ---- clusters and CTA pairs -----------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of the same shared-memory location in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Arrive (release, cluster scope) on an mbarrier of any CTA in the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Non-blocking 4-byte store into another CTA's shared memory whose completion performs
// complete_tx(4) on that CTA's mbarrier; the complete-tx has release semantics at cluster
// scope, so it publishes this thread's prior writes (and those it acquired) to a waiter
// that acquires the barrier, without stalling the issuing thread the way a fenced
// remote arrive does.
__device__ __forceinline__ void st_async_signal(uint32_t remote_word, uint32_t value, uint32_t remote_bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.u32 [%0], %1, [%2];" ::"r"(remote_word),
               "r"(value), "r"(remote_bar)
               : "memory");
}

// try_wait with acquire at cluster scope (barriers that peers or pair commits arrive on).
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded cluster-scope wait; `sleep_ns` > 0 backs off between polls (long waits).
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, const WaitCtl &c,
                                                  uint32_t sleep_ns = 0) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (;;) {
#pragma unroll 1
    for (int i = 0; i < 8; ++i) {
      if (mbar_try_wait_cluster(bar, parity)) return true;
      if (sleep_ns) __nanosleep(sleep_ns);
    }
    if (*c.abort) return false;
    if (globaltimer() - t0 > c.limit_ns) {
      raise_timeout(c);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait_drain_cluster(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer();
  for (;;) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (globaltimer() - t0 > limit_ns) return false;
  }
}

// ---- tcgen05, CTA pair (cta_group::2) ------------------------------------------------
// Both CTAs of the pair execute alloc / relinquish / dealloc from the same warp.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
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
// Pair MMA, A and B from shared memory (each CTA supplies its A rows and its half of B).
template <bool kTF32>
__device__ __forceinline__ void mma_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  if constexpr (kTF32) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
  }
}
// Pair MMA, A from tensor memory (each CTA's own TMEM, same address), B from shared memory.
__device__ __forceinline__ void mma_ts_pair_tf32(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the mbarrier at `bar` in every CTA of `cta_mask` when all pair MMAs
// issued so far by this thread have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}

// 32 lanes x 32 consecutive columns from registers: thread t writes lane (base lane + t).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]),
      "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 16 consecutive columns.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ---- descriptors --------------------------------------------------------------------
// Shared-memory matrix descriptor (sm_100): start >> 4 in [0,14), leading byte offset
// >> 4 in [16,30), stride byte offset >> 4 in [32,46), version 1 at bit 46, swizzle
// mode in [61,64) (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                              uint32_t swizzle) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)swizzle << 61);
}

// One CTA's MN-major B tile: 128 columns x (128 / ELEM) k-rows, ELEM-byte elements, 128-B
// swizzle (TF32: the 32-B-atom form).  The swizzle atom is 128 B of columns x kRows k-rows
// (TF32 32 columns x 4 rows = 512 B, BF16 64 x 8 = 1 KB).  Two tilings of those atoms:
//   column blocks (atoms = false): each 128-B column block holds all of the tile's k-rows,
//     atoms along K one atom apart, blocks (128 / ELEM) x 128 B apart -- one 2-D TMA box per
//     block;
//   k-group major (atoms = true): the column blocks' atoms of one k-group sit side by side
//     (one atom apart), k-groups (128 / (128 / ELEM)) atoms apart -- one 4-D TMA box
//     (columns in block, rows in group, blocks, groups) per tile.
// Same bytes, same results; the tensor core reads the k-group-major tiling faster (TF32 mbr
// 4096^3 671 -> 763 TFLOP/s on the persistent pair kernel).  The descriptor's leading byte
// offset is the stride between column blocks, its stride byte offset that between k-groups.
template <int ELEM>
struct BTileMN {
  static constexpr int kBK = 128 / ELEM, kUmmaK = 32 / ELEM, kNBlk = 128 / ELEM, kBlocks = 128 / kNBlk;
  static constexpr int kRows = ELEM == 4 ? 4 : 8;  // k-rows per atom
  static constexpr uint32_t kAtom = kRows * 128, kSwz = ELEM == 4 ? 1u : 2u;
  // Bytes between k-steps (kUmmaK k-rows).
  __host__ __device__ static constexpr uint32_t step(bool atoms) {
    return atoms ? (kUmmaK / kRows) * kBlocks * kAtom : kUmmaK * 128;
  }
  // Descriptor of k-step ks of the tile at `tile`.
  __device__ __forceinline__ static uint64_t desc(uint32_t tile, int ks, bool atoms) {
    return atoms ? smem_desc(tile + ks * step(true), kAtom, kBlocks * kAtom, kSwz)
                 : smem_desc(tile + ks * step(false), kBK * 128, kAtom, kSwz);
  }
};

// Instruction descriptor for kind::tf32 / kind::f16: D f32 (bit 4), A/B format in [7,10)
// and [10,13) (1 = bf16, 2 = tf32), A K-major (bit 15 = 0), B MN-major (bit 16 = 1),
// N >> 3 in [17,23), M >> 4 in [24,29).
__host__ __device__ constexpr uint32_t instr_desc(uint32_t fmt, uint32_t m, uint32_t n) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (0u << 15) | (1u << 16) | ((n >> 3) << 17) |
         ((m >> 4) << 24);
}
// The same with the majors exchanged: A MN-major (bit 15 = 1), B K-major (bit 16 = 0).
__host__ __device__ constexpr uint32_t instr_desc_a_mn(uint32_t fmt, uint32_t m, uint32_t n) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 15) | (0u << 16) | ((n >> 3) << 17) |
         ((m >> 4) << 24);
}

// Two f32 values rounded to nearest-even bf16, packed: lo in bits [0, 16), hi in [16, 32).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t d;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  return d;
}

// IEEE-2019 maximum(x, +0.0): a NaN input is returned unchanged (payload kept, as the
// reference's fold keeps 0x7FC00000, test/Transforms/canonicalize.mlir:90-100), -0.0 and
// negatives give +0.0.  One ordered compare and a select, in PTX so that it is not
// contracted into a max instruction (which would return the canonical NaN): x <= 0 is
// false for a NaN, which is kept, and true for -0.0, which becomes +0.0.
__device__ __forceinline__ float relu_ieee(float x) {
  float y;
  asm("{\n\t.reg .pred p;\n\tsetp.le.f32 p, %1, 0f00000000;\n\tselp.f32 %0, 0f00000000, %1, p;\n\t}"
      : "=f"(y)
      : "f"(x));
  return y;
}

// ---- 3xTF32 operand split -----------------------------------------------------------
// Round split: hi = tf32_rna(x), lo = tf32_rna(x - hi); the tensor core reads both exactly.
// Truncation split, for tensor cores that read an f32 operand as TF32 by discarding its
// low 13 mantissa bits: hi is x itself (read as trunc(x)), lo = x - trunc(x), which is
// exact in f32 and is read truncated to 11 significant bits.  Non-finite x: lo = 0, and a
// NaN whose payload lies only in the low 13 bits gets its quiet bit set so it is not read
// as an infinity.
__device__ __forceinline__ float split_lo_trunc(float x) {
  const uint32_t u = __float_as_uint(x);
  return ((u & 0x7F800000u) == 0x7F800000u) ? 0.0f : __fsub_rn(x, __uint_as_float(u & 0xFFFFE000u));
}
// Truncation split of four elements on the fast path (2 ops each); `special` reports a
// non-finite element (exponent all ones), which the caller redoes element by element.
__device__ __forceinline__ float4 split_lo_trunc4(const float4 x, bool &special) {
  const uint32_t ux = __float_as_uint(x.x), uy = __float_as_uint(x.y), uz = __float_as_uint(x.z),
                 uw = __float_as_uint(x.w);
  constexpr uint32_t kExp = 0x7F800000u;
  special = max(max(ux & kExp, uy & kExp), max(uz & kExp, uw & kExp)) == kExp;
  return make_float4(__fsub_rn(x.x, __uint_as_float(ux & 0xFFFFE000u)),
                     __fsub_rn(x.y, __uint_as_float(uy & 0xFFFFE000u)),
                     __fsub_rn(x.z, __uint_as_float(uz & 0xFFFFE000u)),
                     __fsub_rn(x.w, __uint_as_float(uw & 0xFFFFE000u)));
}
__device__ __forceinline__ uint32_t split_hi_trunc_bits(uint32_t u) {
  return ((u & 0x7FFFFFFFu) > 0x7F800000u) ? (u | 0x00400000u) : u;
}

// Round-to-nearest (ties away) to tf32: the result is an f32 with the low 13 bits zero.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

}  // namespace tf
