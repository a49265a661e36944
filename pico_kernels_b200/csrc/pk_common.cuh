// Device-side building blocks shared by the sm_100a kernels: shared-memory
// barriers with bounded waits, TMA tile loads, tcgen05 (TMEM + UMMA) wrappers
// and the smem matrix descriptors the tensor core reads.
//
// Every wait in this library is bounded: a wait that does not complete within
// the wait limit (pk_set_wait_limit_ns; by default PK_WAIT_CYCLES SM cycles,
// ~2 s) records PK_ERR_TIMEOUT in the device status word and returns false,
// and the caller unwinds (frees TMEM, returns) instead of spinning forever.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "pk_internal.h"

#ifndef PK_WAIT_CYCLES
#define PK_WAIT_CYCLES 4000000000ll  // ~2 s at 1.9 GHz; legitimate waits are microseconds
#endif

namespace pk {

// ---------------------------------------------------------------------------
// status word
// ---------------------------------------------------------------------------
__device__ __forceinline__ void record_error(int* status, int code, int where) {
  if (status != nullptr) {
    if (atomicCAS(status, 0, code) == 0) status[1] = where;
  }
}

// Wait limit in SM cycles: the 64-bit word after the status code and site
// (pk_set_wait_limit_ns), or PK_WAIT_CYCLES when it is 0 or there is no
// status word. Read only once a wait did not complete on its first probe.
__device__ __forceinline__ long long wait_limit(const int* status) {
  if (status != nullptr) {
    const long long v = *reinterpret_cast<const volatile long long*>(status + 2);
    if (v > 0) return v;
  }
  return PK_WAIT_CYCLES;
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` to complete, for at most the wait limit
// (SM clock cycles; about 2 s at full clock by default). The bound is checked on the SM's
// own cycle counter: cheap to read, unlike the global timer.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int where) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const long long t0 = clock64();
  const long long limit = wait_limit(status);
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(a, parity)) return true;
    if (clock64() - t0 > limit) {
      record_error(status, PK_ERR_TIMEOUT, where);
      return false;
    }
  }
}

// As mbar_wait, but each probe lets the hardware suspend the warp for up to
// `hint_ns` nanoseconds (it resumes as soon as the phase completes), so a
// waiting warp does not spin and take issue slots from working warps.
__device__ __forceinline__ bool mbar_try_wait_hint(uint32_t bar_addr, uint32_t parity,
                                                   uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar_addr), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, int* status,
                                                int where, uint32_t hint_ns = 20000) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  const long long t0 = clock64();
  const long long limit = wait_limit(status);
  while (true) {
    if (mbar_try_wait_hint(a, parity, hint_ns)) return true;
    if (clock64() - t0 > limit) {
      record_error(status, PK_ERR_TIMEOUT, where);
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// programmatic dependent launch and thread-block clusters
// ---------------------------------------------------------------------------
// Wait until the grids this one depends on have completed and their memory
// is visible (a no-op when the launch had no programmatic dependency).
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
// Allow the next grid in the stream (launched with programmatic serialization)
// to start its prologue; it still waits for this grid in griddep_wait().
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// All threads of all CTAs in the cluster; release/acquire orders shared
// memory writes before the barrier with distributed-shared reads after it.
__device__ __forceinline__ void cluster_sync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Explicit shared-memory accesses by 32-bit shared address: a generic pointer
// into shared memory that the compiler cannot trace back compiles to generic
// loads, which take the longer L1TEX path. Loads are volatile so they stay
// after the (volatile) mbarrier wait that publishes the data; stores carry a
// memory clobber.
__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint64_t lds_u64(uint32_t addr) {
  uint64_t v;
  asm volatile("ld.shared.u64 %0, [%1];" : "=l"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint4 lds_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ void sts_u64(uint32_t addr, uint64_t v) {
  asm volatile("st.shared.u64 [%0], %1;" ::"r"(addr), "l"(v) : "memory");
}
__device__ __forceinline__ void sts_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void sts_v4f(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// Named barrier over `nthreads` threads (a multiple of 32) of this CTA.
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (TMA engine and tensor core).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA (tiled bulk tensor copies global -> shared)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0,
                                            int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// Bring a tile into L2 only (no shared-memory destination, no completion).
// A hint: it never changes what a later load returns.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* m, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void tma_load_2d_hint(void* dst, const CUtensorMap* m, uint64_t* bar,
                                                 int c0, int c1, uint64_t hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(hint)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}

__device__ __forceinline__ void tma_store_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void tma_store_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void tma_store_wait_all() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// 16-byte streaming load that bypasses L1 (read-only data read once).
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// L2 eviction-priority hints (createpolicy), used as TMA cache hints.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory and the 5th-generation MMA
// ---------------------------------------------------------------------------
// Allocate `ncols` TMEM columns (power of two >= 32); whole warp executes.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// ---------------------------------------------------------------------------
// CTA-pair (cta_group::2) forms. A cluster of two CTAs shares one MMA: rank 0
// issues it, each CTA holds half of A's rows and half of B's columns in its
// own shared memory at the same offset, and rows 128 r .. 128 r + 127 of D
// land in the TMEM of CTA r. Every tcgen05 instruction of a kernel that uses
// these carries cta_group::2.
// ---------------------------------------------------------------------------
// One warp of EACH CTA of the pair executes the allocation (collectively);
// both CTAs receive the same column base.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// TMA load into this CTA's shared memory, completion signalled on an mbarrier
// of either CTA of the pair (`bar_cluster` is a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m,
                                                 uint32_t bar_cluster, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_f8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at `bar`'s offset in BOTH CTAs of the pair when
// all previously issued pair MMAs of this thread have finished.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// Arrive on an mbarrier of any CTA of the cluster (shared::cluster address).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster)
               : "memory");
}

// mbar_wait with cluster-scope acquire, for phases completed by arrivals from
// the other CTA of the cluster.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* status,
                                                  int where) {
  const uint32_t a = smem_u32(bar);
  const long long t0 = clock64();
  const long long limit = wait_limit(status);
  while (true) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity)
        : "memory");
    if (ok) return true;
    if (clock64() - t0 > limit) {
      record_error(status, PK_ERR_TIMEOUT, where);
      return false;
    }
  }
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]; 16-bit inputs, fp32 accumulate.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Same with 8-bit (e4m3) inputs.
__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once all previously issued tcgen05.mma of this thread finish.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 TMEM lanes x 32 bit, 16 consecutive columns per lane.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 TMEM lanes x 32 bit, 32 consecutive columns per lane.
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
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

// ---------------------------------------------------------------------------
// UMMA shared-memory matrix descriptor (sm_100 format).
//   bits  0-13 start address >> 4
//   bits 16-29 leading-dimension byte offset >> 4
//   bits 32-45 stride-dimension byte offset >> 4
//   bits 46-47 descriptor version (1 on sm_100)
//   bits 61-63 layout: 0 none, 2 = 128-byte swizzle
// K-major, 128B swizzle: rows of 128 B, 8-row groups SBO apart (LBO unused).
// MN-major, 128B swizzle: 128 B along MN x 8 K rows per atom; atoms along MN
// are LBO apart, 8-row K groups SBO apart.
// ---------------------------------------------------------------------------
constexpr uint64_t kDescSwizzle128 = 2;

__device__ __forceinline__ uint64_t make_smem_desc(uint32_t smem_addr, uint32_t lbo_bytes,
                                                   uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= kDescSwizzle128 << 61;
  return d;
}

// Instruction descriptor for kind::f16 / kind::f8f6f4 with fp32 accumulate.
//   bits 4-5 D format (1 = f32), 7-9 A format, 10-12 B format,
//   bit 15 A MN-major, bit 16 B MN-major, 17-22 N>>3, 24-28 M>>4.
// A/B format: kind::f16 -> 0 f16, 1 bf16; kind::f8f6f4 -> 0 e4m3.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_format, bool a_mn_major,
                                                  bool b_mn_major, int m, int n) {
  return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | ((static_cast<uint32_t>(n) >> 3) << 17) |
         ((static_cast<uint32_t>(m) >> 4) << 24);
}

// ---------------------------------------------------------------------------
// int4 -> 16-bit dequant helpers.
// A packed byte holds column 2j in its low nibble and 2j+1 in its high nibble
// (two's complement). Flipping the nibble's sign bit and OR-ing it into the
// mantissa of 128.0 (bf16 0x4300) gives 136 + q exactly; subtracting 136
// yields q. For fp16 the base is 1024.0 (0x6400) and the offset 1032.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
  // (a & b) ^ c; LUT = f(0xF0, 0xCC, 0xAA) = (0xF0 & 0xCC) ^ 0xAA = 0x6A
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

template <typename T>
struct Int4Magic;
template <>
struct Int4Magic<__nv_bfloat16> {
  static constexpr uint32_t kOr = 0x43084308u;   // 128.0 | flipped sign bit, both halves
  static constexpr uint32_t kBias = 0x43084308u; // 136.0 in both halves
};
template <>
struct Int4Magic<__half> {
  static constexpr uint32_t kOr = 0x64086408u;   // 1024.0 | flipped sign bit
  static constexpr uint32_t kBias = 0x64086408u; // 1032.0
};

__device__ __forceinline__ uint32_t sub2(uint32_t a, uint32_t b, __nv_bfloat16*) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t sub2(uint32_t a, uint32_t b, __half*) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b, __nv_bfloat16*) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b, __half*) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Convert one 32-bit word of packed int4 (columns c0..c7 of one K row) into
// exact 16-bit integer codes, four pairs in the order (c0,c4) (c1,c5) (c2,c6)
// (c3,c7): the lanes of a 16-byte chunk hold columns 0,4,1,5,2,6,3,7, a fixed
// permutation the consumer undoes. 3 shifts, 4 lop3 and 4 packed subtracts.
template <typename T>
__device__ __forceinline__ void int4_codes8(uint32_t w, uint32_t (&out)[4]) {
  constexpr uint32_t kMask = 0x000F000Fu;
  T* tag = nullptr;
  out[0] = sub2(lop3_and_xor(w, kMask, Int4Magic<T>::kOr), Int4Magic<T>::kBias, tag);
  out[1] = sub2(lop3_and_xor(w >> 4, kMask, Int4Magic<T>::kOr), Int4Magic<T>::kBias, tag);
  out[2] = sub2(lop3_and_xor(w >> 8, kMask, Int4Magic<T>::kOr), Int4Magic<T>::kBias, tag);
  out[3] = sub2(lop3_and_xor(w >> 12, kMask, Int4Magic<T>::kOr), Int4Magic<T>::kBias, tag);
}

// Column (0..7) held by lane j of a chunk written by int4_codes8.
__host__ __device__ constexpr int int4_codes8_column(int j) { return (j >> 1) + 4 * (j & 1); }

// Dequantize one 32-bit word of packed int4 (8 consecutive columns c0..c7 of
// one K row) into four 16-bit pairs (c0,c1) (c2,c3) (c4,c5) (c6,c7), each
// multiplied by the matching scale pair s01, s23, s45, s67 (same type T).
// With kScaled = false the codes are returned unscaled (exact integers).
template <typename T, bool kScaled>
__device__ __forceinline__ void dequant8(uint32_t w, uint32_t s01, uint32_t s23, uint32_t s45,
                                         uint32_t s67, uint32_t (&out)[4]) {
  constexpr uint32_t kMask = 0x000F000Fu;
  // pairs (c0,c4) (c1,c5) (c2,c6) (c3,c7), biased by +kBias
  uint32_t x04 = lop3_and_xor(w, kMask, Int4Magic<T>::kOr);
  uint32_t x15 = lop3_and_xor(w >> 4, kMask, Int4Magic<T>::kOr);
  uint32_t x26 = lop3_and_xor(w >> 8, kMask, Int4Magic<T>::kOr);
  uint32_t x37 = lop3_and_xor(w >> 12, kMask, Int4Magic<T>::kOr);
  // regroup into adjacent-column pairs
  uint32_t p01 = prmt(x04, x15, 0x5410);
  uint32_t p45 = prmt(x04, x15, 0x7632);
  uint32_t p23 = prmt(x26, x37, 0x5410);
  uint32_t p67 = prmt(x26, x37, 0x7632);
  T* tag = nullptr;
  p01 = sub2(p01, Int4Magic<T>::kBias, tag);
  p23 = sub2(p23, Int4Magic<T>::kBias, tag);
  p45 = sub2(p45, Int4Magic<T>::kBias, tag);
  p67 = sub2(p67, Int4Magic<T>::kBias, tag);
  if constexpr (kScaled) {
    p01 = mul2(p01, s01, tag);
    p23 = mul2(p23, s23, tag);
    p45 = mul2(p45, s45, tag);
    p67 = mul2(p67, s67, tag);
  }
  out[0] = p01;
  out[1] = p23;
  out[2] = p45;
  out[3] = p67;
}

// ---------------------------------------------------------------------------
// Fused output exchange of an N-sharded layer: every rank's kernel stores its
// column slice into all ranks' output buffers (plain peer stores over NVLink;
// no multicast object), then one flag barrier per call. `P` has the fields
// world, rank, peer_flag[] (8-byte aligned words: the arrival count, then,
// for this rank only, its expected count) and done (a zeroed per-grid CTA
// completion counter).
// ---------------------------------------------------------------------------
constexpr int kMaxPeers = 8;

__device__ __forceinline__ void store_elem(void* out, int out_dtype, int64_t idx, float v) {
  if (out_dtype == PK_BF16)
    static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(v);
  else
    static_cast<float*>(out)[idx] = v;
}

// Output element idx (row-major in the local slice's coordinates, leading
// dimension ldo): to `out`, or for a sharded call to idx + n_offset of every
// rank's buffer.
__device__ __forceinline__ void emit_out(void* out, const OutputShard& x, int out_dtype,
                                         int64_t idx, float v) {
  if (x.world == 0) {
    store_elem(out, out_dtype, idx, v);
    return;
  }
  for (int r = 0; r < x.world; ++r)
    store_elem(reinterpret_cast<void*>(x.peer_out[r]), out_dtype, idx + x.n_offset, v);
}

// Called by every thread of each CTA that arrives, after its output stores;
// `arrivals` CTAs of the grid arrive in all (every CTA, or one per cluster
// when a cluster barrier has already ordered its CTAs' stores before the
// leader's). The CTA's peer stores are ordered before one system-scope fence
// by thread 0 through the barrier (the grid-synchronisation pattern), taken
// only by CTAs that stored; the last of the `arrivals` CTAs adds 1 to each
// peer's flag and waits, bounded, until its own flag reaches its next
// expected count, advanced in device memory so CUDA graph replays stay in
// step. The additions are one release pattern: a single system-scope fence,
// then relaxed reductions issued back to back. (A release reduction per peer
// fences before each one, so every peer cost one more NVLink round trip.)
template <typename P>
__device__ __forceinline__ void peer_exchange_finish(const P& p, bool stored, int* status,
                                                     int where, unsigned arrivals) {
  const bool any = __syncthreads_or(stored) != 0;
  if (threadIdx.x + threadIdx.y + threadIdx.z != 0) return;
  if (any) __threadfence_system();
  const unsigned total = arrivals;
  unsigned prev;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(prev) : "l"(p.done) : "memory");
  if (prev != total - 1) return;
  *p.done = 0u;  // re-arm; the next call starts after this grid completes
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int r = 0; r < p.world; ++r) {
    if (r == p.rank) continue;
    asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(p.peer_flag[r]) : "memory");
  }
  unsigned* expected = reinterpret_cast<unsigned*>(p.peer_flag[p.rank]) + 1;
  const uint32_t target = *expected + static_cast<uint32_t>(p.world - 1);
  *expected = target;
  const unsigned* own = reinterpret_cast<const unsigned*>(p.peer_flag[p.rank]);
  const long long t0 = clock64();
  const long long limit = wait_limit(status);
  while (true) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(own) : "memory");
    if (static_cast<int>(v - target) >= 0) break;
    if (clock64() - t0 > limit) {
      record_error(status, PK_ERR_TIMEOUT, where);
      break;
    }
    __nanosleep(100);
  }
}

}  // namespace pk
