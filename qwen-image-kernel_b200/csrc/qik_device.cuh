// qik_device.cuh -- sm_100a device primitives shared by the qik kernels.
//
// Thin inline-PTX wrappers for mbarriers, TMA (cp.async.bulk.tensor), and the
// 5th-generation tensor core (tcgen05: TMEM alloc, MMA, commit, TMEM loads).
// Every wait is bounded: after QIK_WAIT_NS nanoseconds of %globaltimer the wait
// gives up, records QIK_DEV_TIMEOUT in the kernel's status word and raises the
// CTA-local abort flag so the other roles of the CTA stop waiting too.  No trap,
// no assert: a broken pipeline returns an error status instead of hanging.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef QIK_WAIT_NS
#define QIK_WAIT_NS 2000000000ull  // 2 s: far above any legitimate intra-CTA wait
#endif

#define QIK_DEV_OK 0
#define QIK_DEV_TIMEOUT 1
#define QIK_DEV_BAD_ARGS 2

namespace qik {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

// Bounded wait on `parity` of `bar`.  Returns false (and raises the abort flag,
// and records a timeout in *status) when the wait gave up or another role of the
// CTA has already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* status) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0u) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > QIK_WAIT_NS) {
        *abort_flag = 1;
        if (status) atomicExch(status, QIK_DEV_TIMEOUT);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 2-D tiled load into this CTA's shared memory, completing on `bar` (tx bytes).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* m, int32_t x, int32_t y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* m, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* m, int32_t c0, int32_t c1, int32_t c2,
                                            int32_t c3, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}
// Untiled bulk copy of `bytes` (multiple of 16; both addresses 16-byte aligned) from
// global memory into this CTA's shared memory, completing on `bar` (tx bytes).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// 2-D tiled store from this CTA's shared memory (bulk-group completion); elements
// outside the tensor are not written.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, int32_t x, int32_t y, const void* smem_src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(x), "r"(y), "r"(smem_u32(smem_src))
               : "memory");
}
// The same store with an L2 cache policy (createpolicy) for the written lines.
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap* m, int32_t x, int32_t y, const void* smem_src,
                                                  uint64_t policy) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%1, %2}], [%3], %4;" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(x), "r"(y), "r"(smem_u32(smem_src)), "l"(policy)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most 1 committed bulk group of this thread still reads shared memory.
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {  // whole warp
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, e4m3 x e4m3 -> f32 (kind::f8f6f4).
__device__ __forceinline__ void umma_f8f6f4_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem] * B[smem], bf16 x bf16 -> f32 (kind::f16).
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem], bf16 x bf16 -> f32 (kind::f16, A from TMEM).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05 op issued so far by this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)
// Two CTAs of a cluster issue one tensor-core operation together: M = 256 rows, each
// CTA holding half of A (its 128 rows) and half of B (N/2 rows of the K-major tile)
// at the same shared-memory offset, each CTA's tensor memory holding its 128 rows of
// the accumulator.  One thread of the leader CTA (rank 0) issues the MMAs.  Every
// tcgen05 instruction of a kernel uses the same cta_group, so the pair's kernels use
// only the _cg2 forms below.  No load here uses cluster multicast.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {  // all threads of both CTAs
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Shared-memory address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Arrive on an mbarrier of another CTA of the cluster (release at cluster scope).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait with cluster-scope acquire (arrivals or transaction bytes from the
// peer CTA); same give-up rule as mbar_wait.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  int* status) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 63u) == 0u) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > QIK_WAIT_NS) {
        *abort_flag = 1;
        if (status) atomicExch(status, QIK_DEV_TIMEOUT);
        return false;
      }
    }
  }
}
// 2-D tiled load into this CTA's shared memory whose transaction bytes complete on
// the mbarrier at `bar_cluster_addr` (the leader CTA's barrier; shared::cluster
// address).  Not a multicast load.
__device__ __forceinline__ void tma_load_2d_cg2(void* smem_dst, const CUtensorMap* m, int32_t x, int32_t y,
                                                uint32_t bar_cluster_addr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar_cluster_addr)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_cg2(uint32_t* smem_slot, uint32_t ncols) {  // one warp in each CTA
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_cg2() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_cg2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem of both CTAs] (+)= A . B^T for the pair, e4m3 x e4m3 -> f32, M = 256.
__device__ __forceinline__ void umma_f8f6f4_ss_cg2(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                   uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once the pair's previously issued MMAs complete) on the mbarrier at the
// same shared-memory offset in every CTA of `cta_mask`.
__device__ __forceinline__ void umma_commit_cg2(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM words: thread t of the warp receives lane
// (base_lane + t), columns [col, col + 32).  The wait::ld sits in the same asm
// statement so no use of the registers can be scheduled before it.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
// 32 lanes x 128 (64) columns in one instruction: one TMEM round trip for a whole
// 128-key score row (the P row of a 128-key tile).
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, uint32_t (&r)[128]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, %80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, %96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, %112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127}, [%128];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]),
        "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]),
        "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]),
        "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]),
        "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]),
        "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]),
        "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]),
        "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]),
        "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st64(uint32_t taddr, const uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x64.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, %64};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]),
      "r"(r[32]), "r"(r[33]), "r"(r[34]), "r"(r[35]), "r"(r[36]), "r"(r[37]), "r"(r[38]), "r"(r[39]),
      "r"(r[40]), "r"(r[41]), "r"(r[42]), "r"(r[43]), "r"(r[44]), "r"(r[45]), "r"(r[46]), "r"(r[47]),
      "r"(r[48]), "r"(r[49]), "r"(r[50]), "r"(r[51]), "r"(r[52]), "r"(r[53]), "r"(r[54]), "r"(r[55]),
      "r"(r[56]), "r"(r[57]), "r"(r[58]), "r"(r[59]), "r"(r[60]), "r"(r[61]), "r"(r[62]), "r"(r[63])
      : "memory");
}
// 16 lanes x 2 halves (.16x32bx2): threads 0-15 access lanes l0 .. l0 + 15 (l0 = the
// address's lane field) at columns c .. c + n - 1, threads 16-31 the same lanes at
// columns c + 64 .. c + 63 + n: two threads per lane, each with half of a 128-column
// row.
__device__ __forceinline__ void tmem_ld_2x64(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64], 64;\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_2x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.16x32bx2.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32], 64;\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st_2x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.16x32bx2.x32.b32 [%0], 64, {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]),
      "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 layout, version 1) for a tile stored
// with the 128-byte swizzle: rows of 128 bytes, 8-row (1024 B) swizzle atoms.
//   lbo/sbo in bytes; layout 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // 128-byte swizzle
  return d;
}

// Instruction descriptor, dense, f32 accumulate.  a_fmt/b_fmt: kind::f8f6f4 ->
// 0 = E4M3; kind::f16 -> 1 = BF16.  *_mn: 0 = K-major, 1 = MN-major.
__host__ __device__ constexpr uint32_t idesc_f32acc(uint32_t a_fmt, uint32_t b_fmt, uint32_t a_mn, uint32_t b_mn,
                                                    uint32_t M, uint32_t N) {
  return (1u << 4) | (a_fmt << 7) | (b_fmt << 10) | (a_mn << 15) | (b_mn << 16) | ((N >> 3) << 17) |
         ((M >> 4) << 24);
}

// ---------------------------------------------------------------- launch chaining
// Programmatic dependent launch: a kernel launched with the programmatic stream
// serialization attribute may start while its predecessor in the stream is still
// running; pdl_wait() blocks until the predecessor grid has completed and its
// writes are visible.  pdl_trigger() lets the successor grid be scheduled once
// every CTA of this grid has triggered or exited.  Both are no-ops for kernels
// launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- numerics
// Dynamic activation scale from the fp32 bit pattern of max|x| (fp8.py:24-26 as it
// evaluates on CUDA: a division by a host scalar is a multiplication by its fp32
// reciprocal), and the 1/s the activation cast multiplies by.  Shared by every kernel
// that quantizes activations, so they produce the same bytes.
__device__ __forceinline__ float scale_from_amax_bits(uint32_t bits) {
  const float amax = __uint_as_float(bits);
  float s = amax * (1.0f / 448.0f);
  if (s < 1e-12f) s = 1e-12f;  // NaN compares false and passes through
  return s;
}

// 1/s as the activation cast forms it (fp8.py:39 `1.0 / tl.load(...)`): Triton
// lowers an fp32 division to PTX div.full.f32; QIK_ACT_RECIP_RN selects the
// IEEE round-to-nearest reciprocal instead.
__device__ __forceinline__ float act_inverse(float s) {
#ifdef QIK_ACT_RECIP_RN
  return __frcp_rn(s);
#else
  float r;
  asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(1.0f), "f"(s));
  return r;
#endif
}

// fp32 pair -> e4m3 pair, round to nearest even, saturating to +-448 (NaN -> NaN).
__device__ __forceinline__ uint16_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// e4m3 pair -> f16 pair (exact).
__device__ __forceinline__ uint32_t cvt_e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}
// 2^x on the MUFU unit (PTX ex2.approx.ftz.f32): the base-2 exponential of the
// online softmax, as the reference kernel computes it with tl.exp2.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Packed pairs of fp32 (sm_100 f32x2 arithmetic: one instruction for two lanes of work).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// A bf16x2 word (element 0 in the low half) as an fp32 pair, exactly.
__device__ __forceinline__ uint64_t bf2_to_f2(uint32_t w) {
  return f2_pack(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}
// An fp32 pair rounded to nearest even into a bf16x2 word (element 0 in the low half).
__device__ __forceinline__ uint32_t f2_to_bf2(uint64_t v) {
  float lo, hi;
  f2_unpack(v, lo, hi);
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// bf16(silu(g)) of the SwiGLU (triton_fused.py:237-249): g / (1 + e^-g) with the
// reciprocal from rcp.approx (an error of about one fp32 ulp, far below the bf16
// rounding of the result; 1 / inf = 0 gives silu(-large) = -0).  Shared by the SwiGLU
// kernel and the GEMM's SwiGLU epilogue, so both give the same bytes.
__device__ __forceinline__ float silu_bf16(float g) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + __expf(-g)));
  return __bfloat162float(__float2bfloat16_rn(g * r));
}
// bf16x2 product rounded once to nearest even.  The fp32 product of two bf16 values is
// exact (8-bit significands) above the fp32 normal range's floor, so this equals
// bf16(fl32(a) * fl32(b)); only products below 2^-126 (where an fp32 multiply would
// round to a subnormal first) can differ, by the fp32 multiply's double rounding.
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
// bf16x2 sum rounded once to nearest even: for bf16 operands this equals
// bf16(fl32(a) + fl32(b)) (the fp32 sum is exact unless the exponents differ by more
// than 16, and then the smaller operand is far below half a bf16 ulp of the result).
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ float f2_sum(uint64_t v) {
  float lo, hi;
  f2_unpack(v, lo, hi);
  return lo + hi;
}
// Per-head RMSNorm + RoPE arithmetic (rms_rope_kernel, triton_fused.py:28-69), shared by
// the RMSNorm + RoPE kernel and the fused QKV GEMM's epilogue so both give the same
// bytes.  A head of D elements is summed in groups of 8: each group's squares by
// rms_ss8 (even and odd elements in two fp32 fma chains, then added), the D / 8 group
// sums by an xor butterfly over groups (rms_ss_tree16 restates it for D = 128).
__device__ __forceinline__ float rms_ss8(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3) {
  uint64_t ss2 = 0ull;
  ss2 = ffma2(bf2_to_f2(w0), bf2_to_f2(w0), ss2);
  ss2 = ffma2(bf2_to_f2(w1), bf2_to_f2(w1), ss2);
  ss2 = ffma2(bf2_to_f2(w2), bf2_to_f2(w2), ss2);
  ss2 = ffma2(bf2_to_f2(w3), bf2_to_f2(w3), ss2);
  return f2_sum(ss2);
}
// The value every lane holds after `ss += shfl_xor(ss, o)` for o = 8, 4, 2, 1 over 16
// group sums (fp32 addition is commutative, so lanes i and i ^ o add the same pair).
__device__ __forceinline__ float rms_ss_tree16(const float (&g)[16]) {
  float a[8], b[4];
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = g[i] + g[i + 8];
#pragma unroll
  for (int i = 0; i < 4; ++i) b[i] = a[i] + a[i + 4];
  return (b[0] + b[2]) + (b[1] + b[3]);
}
__device__ __forceinline__ float rms_rstd(float ss, int d, float eps) { return rsqrtf(ss / static_cast<float>(d) + eps); }
// One (even, odd) pair: bf16(x * rstd * w) in fp32 with one rounding, then the rotation
// (e + i o)(c + i s) = e (c, s) + o (-s, c) in fp32, rounded to bf16.
__device__ __forceinline__ uint32_t rms_rope_pair(uint32_t xw, uint64_t rr2, uint64_t w2, uint64_t cs2, uint64_t sc2) {
  const uint32_t nb = f2_to_bf2(fmul2(fmul2(bf2_to_f2(xw), rr2), w2));
  const float ne = __uint_as_float(nb << 16), no = __uint_as_float(nb & 0xFFFF0000u);
  return f2_to_bf2(ffma2(f2_pack(ne, ne), cs2, fmul2(f2_pack(no, no), sc2)));
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}
// 2^x for a pair of x <= 2^7 on the FMA pipe (no MUFU): x = n + f with n = round(x)
// (the 1.5 * 2^23 shifter), 2^f by a cubic in f on [-1/2, 1/2] (coefficients
// fitted for least relative error by tests/exp2_poly.py: max relative error
// 7.5e-5 = 2^-13.7), 2^n added to the exponent bits.  x is clamped to >= -125, so
// inputs below give 2^-125 (not 0): callers use it only where every x belongs to an
// allowed key of a row with a finite running max.
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x2) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  float x0, x1;
  f2_unpack(x2, x0, x1);
  const uint64_t xc = f2_pack(fmaxf(x0, -125.0f), fmaxf(x1, -125.0f));
  const uint64_t r = fadd2(xc, f2_pack(kShift, kShift));      // low mantissa bits = round(x)
  const uint64_t n = fadd2(r, f2_pack(-kShift, -kShift));     // round(x) as a float
  const uint64_t f = ffma2(n, f2_pack(-1.0f, -1.0f), xc);      // x - round(x), exact
  uint64_t p = ffma2(f, f2_pack(0x1.c3f748p-5f, 0x1.c3f748p-5f), f2_pack(0x1.f0de1ap-3f, 0x1.f0de1ap-3f));
  p = ffma2(p, f, f2_pack(0x1.62f31ap-1f, 0x1.62f31ap-1f));
  p = ffma2(p, f, f2_pack(0x1.fff692p-1f, 0x1.fff692p-1f));
  // per half: bits(p) + (bits(r) << 23), where (bits(r) << 23) == round(x) << 23
  // modulo 2^32 (the shifter's own bits leave the word); 32-bit adds, one per half
  uint32_t r0, r1, p0, p1;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(r0), "=r"(r1) : "l"(r));
  asm("mov.b64 {%0, %1}, %2;" : "=r"(p0), "=r"(p1) : "l"(p));
  uint64_t out;
  asm("mov.b64 %0, {%1, %2};" : "=l"(out) : "r"(p0 + (r0 << 23)), "r"(p1 + (r1 << 23)));
  return out;
}
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Eight bf16 (one 16-byte vector) -> eight e4m3 codes of fl32(x) * inv: the activation
// cast (fp8.py:36-41).  Returns bytes 0-3, bytes 4-7 in hi_word.
__device__ __forceinline__ uint32_t pack8_e4m3(const uint4 a, float inv, uint32_t& hi_word) {
  const uint32_t w[4] = {a.x, a.y, a.z, a.w};
  const uint64_t inv2 = f2_pack(inv, inv);
  uint32_t o[2];
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    float a0, a1, b0, b1;
    f2_unpack(fmul2(bf2_to_f2(w[2 * j]), inv2), a0, a1);  // each lane an fp32 multiply, as fl32(x) * inv
    f2_unpack(fmul2(bf2_to_f2(w[2 * j + 1]), inv2), b0, b1);
    o[j] = static_cast<uint32_t>(cvt_e4m3x2(a0, a1)) | (static_cast<uint32_t>(cvt_e4m3x2(b0, b1)) << 16);
  }
  hi_word = o[1];
  return o[0];
}

// ---------------------------------------------------------------- L2 cache policies
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint4 ld_nc_hint(const uint4* p, uint64_t pol) {
  uint4 r;
  asm volatile("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ void st_v2_hint(void* p, uint32_t a, uint32_t b, uint64_t pol) {
  asm volatile("st.global.L2::cache_hint.v2.b32 [%0], {%1, %2}, %3;" ::"l"(p), "r"(a), "r"(b), "l"(pol) : "memory");
}
// bulk_load with an L2 cache policy for the source lines.
__device__ __forceinline__ void bulk_load_hint(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar,
                                               uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// ---------------------------------------------------------------- grid-wide amax
// Workspace of the kernels that must know max|x| over the whole tensor before they
// write a single e4m3 code (the single-pass activation quantizer, the layer norm that
// emits codes).  `bar` is a grid barrier: a generation in the high 32 bits and the
// arrivals of the running call in the low 32.  The last CTA to arrive returns the
// arrivals to 0 and advances the generation in one atomic add, so a workspace that
// was zeroed once serves any number of calls in stream order without being cleared
// again.  partial[i] holds CTA i's max|x| bits for the running call: written before
// the CTA arrives, read by every CTA after the barrier, so stale contents never
// matter.  amax_bits belongs to the two-pass form (amax kernel, then pack), which
// clears it itself.  Kernels using the barrier are launched cooperatively (every CTA
// resident), with at most kQuantMaxCtas CTAs.
constexpr int kQuantMaxCtas = 252;
struct QuantWs {
  unsigned long long bar;
  uint32_t amax_bits;
  uint32_t pad;
  uint32_t partial[kQuantMaxCtas];
};
static_assert(sizeof(QuantWs) == 1024, "QuantWs layout");
constexpr uint32_t kQuantAbortMark = 0xFFFFFFFFu;  // a partial above every |x| bit pattern: a CTA gave up

// One thread per CTA: publish this CTA's max (bits; kQuantAbortMark when the CTA gave
// up) in its slot and wait until every CTA of the grid has published.  The arrival
// releases the slot write; the last arrival acquires every earlier one (they form one
// release sequence) and publishes the next generation.  Returns false when the wait
// ran out (QIK_WAIT_NS).
__device__ __forceinline__ bool grid_max_publish_wait(QuantWs* ws, uint32_t m) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(&ws->partial[blockIdx.x]), "r"(m) : "memory");
  unsigned long long old;
  asm volatile("atom.add.acq_rel.gpu.global.u64 %0, [%1], 1;" : "=l"(old) : "l"(&ws->bar) : "memory");
  const uint32_t gen = static_cast<uint32_t>(old >> 32);
  if (static_cast<uint32_t>(old) == gridDim.x - 1) {
    const unsigned long long step = (1ull << 32) - gridDim.x;  // generation + 1, arrivals back to 0
    asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(&ws->bar), "l"(step) : "memory");
    return true;
  }
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0;; ++it) {
    unsigned long long cur;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(cur) : "l"(&ws->bar) : "memory");
    if (static_cast<uint32_t>(cur >> 32) != gen) return true;
    if ((it & 255u) == 255u && globaltimer() - t0 > QIK_WAIT_NS) return false;
  }
}
// One full warp, after its CTA passed grid_max_publish_wait: the max over every CTA's
// slot (kQuantAbortMark when any CTA gave up), in every lane.
// All of a lane's slot loads are issued before the first is used, so the collect costs
// one L2 round trip rather than one per 32 slots.
__device__ __forceinline__ uint32_t grid_max_collect(const QuantWs* ws) {
  constexpr int kPerLane = (kQuantMaxCtas + 31) / 32;
  const uint32_t lane = threadIdx.x & 31u;
  uint32_t v[kPerLane];
#pragma unroll
  for (int k = 0; k < kPerLane; ++k) {
    const uint32_t i = lane + 32u * static_cast<uint32_t>(k);
    v[k] = 0u;
    if (i < gridDim.x) asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v[k]) : "l"(&ws->partial[i]) : "memory");
  }
  uint32_t g = 0;
#pragma unroll
  for (int k = 0; k < kPerLane; ++k) g = max(g, v[k]);
  return __reduce_max_sync(0xffffffffu, g);
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace qik
