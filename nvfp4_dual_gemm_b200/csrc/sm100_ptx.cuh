// sm100_ptx.cuh — thin inline-PTX helpers for sm_100a: mbarriers with bounded
// waits, TMA tensor / bulk copies, tcgen05 (TMEM alloc, copy, block-scaled
// MMA, commit, load) and the shared-memory / instruction descriptors.
//
// Written from the PTX ISA description of each instruction.  The reference
// keeps equivalent wrappers in tcgen05-interface.cuh and tma-interface.cuh;
// the differences that matter here: every wait is bounded by %clock64 and
// reports through a device error word instead of spinning forever
// (tma-interface.cuh:64-75 spins unbounded), and the TMEM base address
// returned by tcgen05.alloc is always used instead of being assumed to be 0.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace nvfp4dg {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Orders this thread's earlier (generic-proxy) view of global memory before
// its later bulk copies (async proxy) that read it.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Time limit of every wait in the kernels of this library, in SM clock
// cycles (about 1-2.5 s between the 1965 MHz boost clock and the ~1.3 GHz
// power-capped clock).  A legitimate wait lasts microseconds; the limit only
// exists so that a logic error ends the kernel with an error word instead of
// hanging the GPU.  The SM-local %clock64 is used because it is a register
// read; %globaltimer is a slow memory-mapped read that, taken on every missed
// poll, serialised the whole pipeline.
constexpr long long kWaitLimitCycles = 2500ll * 1000ll * 1000ll;

__device__ __forceinline__ long long clock_cycles() {
  long long t;
  asm volatile("mov.u64 %0, %%clock64;" : "=l"(t));
  return t;
}

// Set (to 1) in a CTA when one of its bounded waits gives up; cleared by the
// kernels' barrier initialisation before any wait.  A CTA that gave up may
// not have awaited every signal its cluster peers send it, so it lingers
// before leaving (see linger_if_wait_failed).
__shared__ unsigned s_wait_failed;

__device__ __forceinline__ void note_wait_failed() {
  *reinterpret_cast<volatile unsigned*>(&s_wait_failed) = 1u;
}

// Wait until the phase with parity `parity` of `bar` has completed.  Returns
// false (after setting `code` in *err) if the time limit expires, or early if
// *err is already non-zero because another role gave up.
// With bail_on_err = false the wait ignores *err and only the time limit
// ends it (used to drain copies and MMAs before the CTA exits).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned* err, unsigned code,
                                          bool bail_on_err = true) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = 0;
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 0u) {
      const long long now = clock_cycles();
      if (t0 == 0) {
        t0 = now;
        continue;
      }
      if (bail_on_err && *reinterpret_cast<volatile unsigned*>(err) != 0u) {
        note_wait_failed();
        return false;
      }
      if (now - t0 > kWaitLimitCycles) {
        atomicOr(err, code);
        note_wait_failed();
        return false;
      }
    }
  }
}

// GPU-scope release add and acquire load of a 32-bit counter in global
// memory (stream-K tile counters).
__device__ __forceinline__ void red_release_add(int* ptr, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(ptr), "r"(v)
               : "memory");
}
__device__ __forceinline__ int ld_acquire(const int* ptr) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(ptr)
               : "memory");
  return v;
}

// Wait until the counter at `ptr` reaches `target`, bounded like mbar_wait.
__device__ __forceinline__ bool wait_count(const int* ptr, int target,
                                           unsigned* err, unsigned code,
                                           long long limit = kWaitLimitCycles) {
  if (ld_acquire(ptr) == target) return true;
  const long long t0 = clock_cycles();
  for (;;) {
    __nanosleep(32);
    if (ld_acquire(ptr) == target) return true;
    if (*reinterpret_cast<volatile unsigned*>(err) != 0u) {
      note_wait_failed();
      return false;
    }
    if (clock_cycles() - t0 > limit) {
      atomicOr(err, code);
      note_wait_failed();
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// L2 cache policies (createpolicy) and TMA / bulk copies
// ---------------------------------------------------------------------------
// The 64-bit cache-policy operands of the copies' .L2::cache_hint, as
// constants: the values createpolicy.fractional.L2::<priority>.b64 with
// fraction 1.0 returns on B200 (read back from the instruction; evict_first
// and evict_last are also the CacheHintSm100 values published in CUTLASS's
// cute/arch/copy_sm90_desc.hpp).  Creating them at run time puts that
// instruction's latency on the first copy's path.
constexpr uint64_t kPolicyEvictNormal = 0x16F0000000000000ull;
constexpr uint64_t kPolicyEvictFirst = 0x12F0000000000000ull;
constexpr uint64_t kPolicyEvictLast = 0x14F0000000000000ull;

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m))
               : "memory");
}

// 2-D tiled TMA load global -> this CTA's shared memory; completion is
// signalled as transaction bytes on `bar`.  c0 is the innermost coordinate.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m,
                                            uint64_t* bar, int c0, int c1,
                                            int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_"
      "tx::bytes.L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2),
      "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Contiguous bulk copy global -> shared (16-byte aligned, size % 16 == 0).
__device__ __forceinline__ void bulk_load(void* dst, const void* src,
                                          uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::"
      "cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// L2 prefetches (hints: nothing is written, nothing waits for them).  A
// 2-D box of a tensor map, and a contiguous run (16-byte aligned, size a
// multiple of 16).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* m, int c0,
                                                int c1) {
  asm volatile(
      "cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void bulk_prefetch_l2(const void* src,
                                                 uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src),
               "r"(bytes)
               : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols)
      : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Copy a 32-row x 16-byte block from shared memory (described by `sdesc`)
// into 4 TMEM columns starting at `taddr`, replicated into all four 32-lane
// sub-partitions: lane 32q+i, column c receives bytes [16i + 4c, 16i + 4c + 4).
__device__ __forceinline__ void tc_cp_32x128b_x4(uint32_t taddr,
                                                 uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr),
               "l"(sdesc)
               : "memory");
}

// D(tmem) (+)= A(smem) * B(smem)^T with block scales read from TMEM;
// kind::mxf4nvf4, one e4m3 scale per 16 K elements (scale_vec::4X).
// Collector: kCollNone reads A from shared memory; kCollFill reads it and
// keeps it in the A collector; kCollLastUse takes A from the collector (the
// immediately preceding MMA must have used kCollFill with the same A).
enum Collector : int { kCollNone = 0, kCollFill = 1, kCollLastUse = 2 };

#define NVFP4DG_MMA_ASM(COLL)                                                \
  asm volatile(                                                              \
      "{\n\t.reg .pred p;\n\t"                                               \
      "setp.ne.b32 p, %4, 0;\n\t"                                             \
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.scale_vec::4X" COLL \
      " [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),                  \
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem),  \
      "r"(sfb_tmem)                                                          \
      : "memory")

template <int kColl = kCollNone>
__device__ __forceinline__ void tc_mma_nvf4(uint32_t d_tmem, uint64_t a_desc,
                                            uint64_t b_desc, uint32_t idesc,
                                            uint32_t sfa_tmem,
                                            uint32_t sfb_tmem,
                                            uint32_t accumulate) {
  if constexpr (kColl == kCollFill) {
    NVFP4DG_MMA_ASM(".collector::a::fill");
  } else if constexpr (kColl == kCollLastUse) {
    NVFP4DG_MMA_ASM(".collector::a::lastuse");
  } else {
    NVFP4DG_MMA_ASM("");
  }
}
#undef NVFP4DG_MMA_ASM

// Arrive once on `bar` when all previously issued tcgen05 async operations of
// this thread have completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(smem_u32(bar))
      : "memory");
}

// Each thread of the warp reads 32 consecutive fp32 columns of its TMEM lane.
// 16 consecutive 32-bit TMEM columns of this warp's 32 lanes -> v[0..15].
__device__ __forceinline__ void tc_ld_16cols(uint32_t taddr, float (&v)[16]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tc_ld_32cols(uint32_t taddr, float (&v)[32]) {
  uint32_t* r = reinterpret_cast<uint32_t*>(v);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]),
        "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
        "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
// Each thread of the warp writes N consecutive 32-bit TMEM columns of its
// lane (the warp's 32-lane sub-partition is selected by the lane field of
// taddr).
__device__ __forceinline__ void tc_st_16cols(uint32_t taddr,
                                             const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
      "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
      "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tc_st_32cols(uint32_t taddr,
                                             const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, "
      "%30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]),
      "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]),
      "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16-byte shared-memory load.
__device__ __forceinline__ uint4 lds128(uint32_t saddr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(saddr)
               : "memory");
  return v;
}

__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Marks 32 registers as written here (an empty statement), to be placed
// right after a tcgen05.wait::ld: uses of the registers a tcgen05.ld fills
// asynchronously are then not scheduled before the wait.
__device__ __forceinline__ void tie32(float (&a)[32]) {
  asm volatile(""
               : "+f"(a[0]), "+f"(a[1]), "+f"(a[2]), "+f"(a[3]), "+f"(a[4]),
                 "+f"(a[5]), "+f"(a[6]), "+f"(a[7]), "+f"(a[8]), "+f"(a[9]),
                 "+f"(a[10]), "+f"(a[11]), "+f"(a[12]), "+f"(a[13]),
                 "+f"(a[14]), "+f"(a[15]), "+f"(a[16]), "+f"(a[17]),
                 "+f"(a[18]), "+f"(a[19]), "+f"(a[20]), "+f"(a[21]),
                 "+f"(a[22]), "+f"(a[23]), "+f"(a[24]), "+f"(a[25]),
                 "+f"(a[26]), "+f"(a[27]), "+f"(a[28]), "+f"(a[29]),
                 "+f"(a[30]), "+f"(a[31])
               :
               : "memory");
}

// ---------------------------------------------------------------------------
// Thread-block clusters and the 2-SM (cta_group::2) forms
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
               : "=r"(r)
               : "r"(saddr), "r"(rank));
  return r;
}

// Cluster-wide execution barrier (every thread of every CTA of the cluster).
// Programmatic dependent launch: wait until the grids this one depends on
// have completed and their memory is visible (a no-op when launched without
// the programmatic attribute), and allow the next grid in the stream to be
// scheduled before this one ends.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Split-phase cluster barrier: every thread of every CTA of the cluster
// arrives (release) and later waits (acquire); a thread must wait before it
// arrives again.
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
// Arrival without memory ordering: for start-up, where the barrier objects
// were already published by fence.mbarrier_init.release.cluster.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) from
// this CTA's shared memory to another CTA's (cluster address); completion is
// counted as transaction bytes on the destination CTA's mbarrier.
__device__ __forceinline__ void bulk_s2s_cluster(uint32_t dst_cluster,
                                                 uint32_t src_cta,
                                                 uint32_t bytes,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(bar_cluster)
      : "memory");
}

__device__ __forceinline__ void sts128(uint32_t saddr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(saddr),
               "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// Final cluster barrier of a kernel in which every signal or copy into a
// peer CTA's shared memory is awaited by that peer before it gets here: the
// arrival needs no release ordering (a release arrival would wait for this
// thread's outstanding global writes, e.g. the C tile stores, to complete).
// A CTA in which a bounded wait gave up may have skipped some of those
// waits; it stays resident for ~50K more cycles (a bounded spin) so that
// anything still in flight towards it lands before its shared memory is
// released.
__device__ __forceinline__ void cluster_sync_final() {
  cluster_arrive_relaxed();
  cluster_wait();
  if (*reinterpret_cast<volatile unsigned*>(&s_wait_failed) != 0u) {
    const long long t0 = clock_cycles();
    while (clock_cycles() - t0 < 50000) {
    }
  }
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::
          : "memory");
}

// Arrive on an mbarrier of any CTA of the cluster (cluster address), with
// the default semantics of mbarrier.arrive.  A cluster-scope release here
// cost 1000-2000 cycles per arrival on B200 (it waits out the SM's memory
// traffic); the producers of the data these arrivals publish (TMEM scale
// stores, TMEM accumulator reads) complete before the arrival
// (tcgen05.wait::st / ::ld) and are ordered for the MMA by the tcgen05
// fences around the barrier, the pattern CUTLASS's 2-SM pipelines use.
// 16-byte store into another CTA's shared memory (cluster address) whose
// completion is counted as 16 transaction bytes on an mbarrier of that CTA.
__device__ __forceinline__ void st_async_v4(uint32_t cluster_addr,
                                            const float (&v)[4],
                                            uint32_t cluster_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], "
      "{%1, %2, %3, %4}, [%5];" ::"r"(cluster_addr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
      "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(cluster_bar)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(
                   cluster_addr)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx_cluster(
    uint32_t cluster_addr, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(
          cluster_addr),
      "r"(bytes)
      : "memory");
}

// Waits on barriers that the peer CTA signals use the ordinary bounded wait.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar,
                                                  uint32_t parity,
                                                  unsigned* err, unsigned code,
                                                  bool bail_on_err = true) {
  return mbar_wait(bar, parity, err, code, bail_on_err);
}

// 2-D tiled TMA load into this CTA's shared memory whose completion bytes
// are counted on an mbarrier of either CTA of the pair (cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m,
                                                 uint32_t bar_cluster, int c0,
                                                 int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::"
      "complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(bar_cluster),
      "l"(policy)
      : "memory");
}

// The same with a third (batch) coordinate, for batched problems (L > 1).
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* m,
                                                 uint32_t bar_cluster, int c0,
                                                 int c1, int c2,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::"
      "complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2),
      "r"(bar_cluster), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem,
                                                uint32_t ncols) {
  asm volatile(
      "tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
          smem_u32(dst_smem)),
      "r"(ncols)
      : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr,
                                                  uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(
                   taddr),
               "r"(ncols)
               : "memory");
}

// 2-SM block-scaled MMA, issued by the even CTA of the pair: each CTA holds
// M/2 rows of A and N/2 rows of B at the same shared-memory offsets, its own
// scale factors in TMEM, and receives its M/2 rows of D.
__device__ __forceinline__ void tc_mma_nvf4_pair(uint32_t d_tmem,
                                                 uint64_t a_desc,
                                                 uint64_t b_desc,
                                                 uint32_t idesc,
                                                 uint32_t sfa_tmem,
                                                 uint32_t sfb_tmem,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.scale_vec::4X "
      "[%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem),
      "r"(sfb_tmem)
      : "memory");
}

// Arrive once on the mbarrier at `bar_cluster` (either CTA of the pair) when
// this thread's previously issued 2-SM tcgen05 operations have completed.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar_cluster) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 "
      "[%0];" ::"r"(bar_cluster)
      : "memory");
}

// ---------------------------------------------------------------------------
// TMA tensor stores (shared -> global), bulk async-group completion
// ---------------------------------------------------------------------------
// 2-D / 3-D tiled store of a box from this CTA's shared memory; the copy
// reads shared memory asynchronously and is tracked by the issuing thread's
// bulk async-group (commit with bulk_commit_group).  Boxes that extend past
// the tensor's bounds are clipped.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m,
                                             const void* src, int c0,
                                             int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], "
      "[%3];" ::"l"(reinterpret_cast<uint64_t>(m)),
      "r"(c0), "r"(c1), "r"(smem_u32(src))
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* m,
                                             const void* src, int c0, int c1,
                                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, "
      "%3}], [%4];" ::"l"(reinterpret_cast<uint64_t>(m)),
      "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until every committed bulk group of this thread has finished reading
// its shared-memory source (the buffer may be rewritten).
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// Wait until every committed bulk group of this thread has completed.
__device__ __forceinline__ void bulk_wait_group0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor (tcgen05 format): start address, leading-
// and stride-dimension byte offsets (all >> 4), the fixed version bits 46-48 =
// 0b001, base offset 0 and the layout (swizzle) type in bits 61-63.
enum class SmemLayout : uint32_t { kNone = 0, kSwizzle128B = 2 };

__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo,
                                              uint32_t sbo, SmemLayout lay) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo & 0x3FFFFu) >> 4) << 16;
  d |= static_cast<uint64_t>((sbo & 0x3FFFFu) >> 4) << 32;
  d |= 1ull << 46;
  d |= static_cast<uint64_t>(lay) << 61;
  return d;
}

// Instruction descriptor for kind::mxf4nvf4: A and B e2m1 (format code 1 in
// bits 7-9 and 10-12), both K-major, dense, N >> 3 in bits 17-22, scale type
// UE4M3 (bit 23 = 0), M >> 4 in bits 24-28, scale-factor ids 0, K = 64.
__host__ __device__ constexpr uint32_t idesc_nvf4(int m, int n) {
  return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

}  // namespace nvfp4dg
