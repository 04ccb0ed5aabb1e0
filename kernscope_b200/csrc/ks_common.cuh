// ks_common.cuh -- shared device/host helpers for the sm_100a kernels:
// status plumbing, bf16 packing, warp/block reductions, bounded mbarrier
// waits, TMA (cp.async.bulk.tensor) and tcgen05 (TMEM alloc, UMMA issue,
// commit, TMEM loads) wrappers written as inline PTX.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernscope_b200.h"

#define KS_DEV __device__ __forceinline__

// ---------------------------------------------------------------------------
// Device error word.  Bounded waits record a code here and return instead of
// spinning forever; the host reads and clears it with ks_device_error_take().
// ---------------------------------------------------------------------------
enum : int {
  KS_DEVERR_NONE = 0,
  KS_DEVERR_WAIT_TIMEOUT = 1,   // an mbarrier wait hit its limit
  KS_DEVERR_SELFTEST = 2,       // the self-test wait (expected)
};

// Passed by value to every kernel that waits: where to record a timeout and
// how long (ns, %globaltimer) a single wait may take.
struct KsWait {
  int *err;
  unsigned long long limit_ns;
};

KS_DEV uint64_t ks_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

KS_DEV void ks_record_error(int *err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// ---------------------------------------------------------------------------
// bf16 helpers
// ---------------------------------------------------------------------------
KS_DEV float ks_bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
KS_DEV float ks_bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
KS_DEV float ks_bf16_to_f32(uint16_t h) { return __uint_as_float(uint32_t(h) << 16); }
// Round-to-nearest-even pack of two floats (lo in the low half).
KS_DEV uint32_t ks_pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&v);
}
KS_DEV uint16_t ks_f32_to_bf16(float f) {
  __nv_bfloat16 v = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t *>(&v);
}

// ---------------------------------------------------------------------------
// Reductions
// ---------------------------------------------------------------------------
KS_DEV float ks_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
KS_DEV float ks_warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
KS_DEV double ks_warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// Shared-memory addresses, mbarriers, fences
// ---------------------------------------------------------------------------
KS_DEV uint32_t ks_smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

KS_DEV void ks_mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(ks_smem_u32(bar)), "r"(count));
}
KS_DEV void ks_fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
KS_DEV void ks_fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

KS_DEV void ks_mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(ks_smem_u32(bar)) : "memory");
}
KS_DEV void ks_mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(ks_smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// Non-blocking test of a phase (never suspends the thread).
KS_DEV bool ks_mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

KS_DEV bool ks_mbar_try_wait(uint32_t bar, uint32_t parity) {
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

// Bounded wait for the phase with the given parity to complete.  Returns
// false (and records KS_DEVERR_WAIT_TIMEOUT) once w.limit_ns has elapsed, or
// at once when *abort is already set by another role of the CTA.
KS_DEV bool ks_mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort, const KsWait &w) {
  const uint32_t a = ks_smem_u32(bar);
  if (ks_mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = ks_globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (ks_mbar_try_wait(a, parity)) return true;
    if (abort != nullptr && *abort) return false;
    if (ks_globaltimer() - t0 > w.limit_ns) {
      ks_record_error(w.err, KS_DEVERR_WAIT_TIMEOUT);
      if (abort != nullptr) *abort = 1;
      return false;
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------
KS_DEV void ks_prefetch_tmap(const CUtensorMap *m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// Untiled bulk copy global -> shared (16-byte aligned addresses, size a
// multiple of 16), completion counted on `bar` in bytes.
KS_DEV void ks_bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   ks_smem_u32(dst)),
               "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(ks_smem_u32(bar))
               : "memory");
}

KS_DEV void ks_tma_load_2d(void *dst, const CUtensorMap *m, uint64_t *bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(ks_smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(ks_smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
KS_DEV void ks_tma_load_3d(void *dst, const CUtensorMap *m, uint64_t *bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(ks_smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(ks_smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// L2 eviction priority for the cache-hinted loads below: lines loaded with
// this policy are evicted after normal ones.
KS_DEV uint64_t ks_l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// The tiled loads above with an L2 cache policy.
KS_DEV void ks_tma_load_2d_hint(void *dst, const CUtensorMap *m, uint64_t *bar, int c0, int c1, uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(ks_smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(ks_smem_u32(bar)), "r"(c0), "r"(c1), "l"(pol)
      : "memory");
}
KS_DEV void ks_tma_load_3d_hint(void *dst, const CUtensorMap *m, uint64_t *bar, int c0, int c1, int c2,
                                uint64_t pol) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(ks_smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(ks_smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "l"(pol)
      : "memory");
}

// TMA store of a 2-D box from this CTA's shared memory (bulk-group
// completion: commit, then wait_group.read before the buffer is rewritten and
// wait_group 0 before exit).  Non-negative coordinates only; the innermost
// coordinate times the element size is a multiple of 16 bytes.
KS_DEV void ks_tma_store_2d(const CUtensorMap *m, const void *src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(ks_smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
KS_DEV void ks_tma_store_3d(const CUtensorMap *m, const void *src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(ks_smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
KS_DEV void ks_bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// At most N committed bulk groups still reading their shared-memory source.
template <int N>
KS_DEV void ks_bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Every committed bulk group complete (its global writes done).
KS_DEV void ks_bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA issue, commit, TMEM <-> register moves
// ---------------------------------------------------------------------------
KS_DEV void ks_tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ks_smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
KS_DEV void ks_tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
KS_DEV void ks_tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
KS_DEV void ks_tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KS_DEV void ks_tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]
KS_DEV void ks_umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
KS_DEV void ks_umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every tcgen05 op issued so far by this thread
// has completed.
KS_DEV void ks_umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   ks_smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (clusters of 2, tcgen05 cta_group::2): one MMA issued by the
// even CTA computes a 256-row tile, each CTA holding 128 rows of A, half of
// the B columns and 128 lanes of the accumulator.  No multicast: every TMA
// load writes only the issuing CTA's shared memory; only its completion
// signal may go to the even CTA's barrier.
// ---------------------------------------------------------------------------
KS_DEV uint32_t ks_cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
KS_DEV uint32_t ks_cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// fp32 load from another CTA's shared memory (address from ks_mapa).
KS_DEV float ks_ld_shared_cluster_f32(uint32_t cluster_addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(cluster_addr) : "memory");
  return v;
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
KS_DEV uint32_t ks_mapa(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
// All threads of all CTAs of the cluster (release / acquire at cluster scope).
KS_DEV void ks_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of any CTA of the cluster (address from ks_mapa).
KS_DEV void ks_mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
KS_DEV bool ks_mbar_try_wait_acq_cluster(uint32_t bar, uint32_t parity) {
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
// ks_mbar_wait for a barrier that receives arrivals from the other CTA.
KS_DEV bool ks_mbar_wait_cluster(uint64_t *bar, uint32_t parity, volatile int *abort, const KsWait &w) {
  const uint32_t a = ks_smem_u32(bar);
  if (ks_mbar_try_wait_acq_cluster(a, parity)) return true;
  const uint64_t t0 = ks_globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (ks_mbar_try_wait_acq_cluster(a, parity)) return true;
    if (abort != nullptr && *abort) return false;
    if (ks_globaltimer() - t0 > w.limit_ns) {
      ks_record_error(w.err, KS_DEVERR_WAIT_TIMEOUT);
      if (abort != nullptr) *abort = 1;
      return false;
    }
  }
}
// TMA load into this CTA's shared memory whose completion (bytes) is counted
// on a barrier that may belong to the other CTA of the pair.
KS_DEV void ks_tma_load_2d_pair(void *dst, const CUtensorMap *m, uint32_t bar_cluster_addr, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(ks_smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster_addr), "r"(c0), "r"(c1)
      : "memory");
}
// TMEM allocation shared by the pair: the same warp of both CTAs executes it.
KS_DEV void ks_tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ks_smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
KS_DEV void ks_tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
KS_DEV void ks_tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Pair MMA (issued by the even CTA only): D[256 x N] (+)= A[256 x K] B[K x N].
KS_DEV void ks_umma_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the barrier at `cluster_addr` (either CTA of the pair) when
// every pair MMA issued so far by this thread has completed.
KS_DEV void ks_umma_commit_pair(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_addr)
               : "memory");
}

KS_DEV void ks_tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
KS_DEV void ks_tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 16 consecutive columns per thread.
KS_DEV void ks_tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 32 bit, 32 consecutive columns per thread.
KS_DEV void ks_tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 32 bit, columns [OFF, OFF+32) of a larger per-thread array
// (elements named directly so the array stays in registers).
template <int OFF, int N>
KS_DEV void ks_tmem_ld32_at(uint32_t taddr, uint32_t (&r)[N]) {
  static_assert(OFF + 32 <= N, "range");
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
               : "=r"(r[OFF + 0]),"=r"(r[OFF + 1]),"=r"(r[OFF + 2]),"=r"(r[OFF + 3]),"=r"(r[OFF + 4]),"=r"(r[OFF + 5]),"=r"(r[OFF + 6]),"=r"(r[OFF + 7]),"=r"(r[OFF + 8]),"=r"(r[OFF + 9]),"=r"(r[OFF + 10]),"=r"(r[OFF + 11]),"=r"(r[OFF + 12]),"=r"(r[OFF + 13]),"=r"(r[OFF + 14]),"=r"(r[OFF + 15]),"=r"(r[OFF + 16]),"=r"(r[OFF + 17]),"=r"(r[OFF + 18]),"=r"(r[OFF + 19]),"=r"(r[OFF + 20]),"=r"(r[OFF + 21]),"=r"(r[OFF + 22]),"=r"(r[OFF + 23]),"=r"(r[OFF + 24]),"=r"(r[OFF + 25]),"=r"(r[OFF + 26]),"=r"(r[OFF + 27]),"=r"(r[OFF + 28]),"=r"(r[OFF + 29]),"=r"(r[OFF + 30]),"=r"(r[OFF + 31])
               : "r"(taddr));
}
template <int OFF, int N>
KS_DEV void ks_tmem_st32_at(uint32_t taddr, const uint32_t (&r)[N]) {
  static_assert(OFF + 32 <= N, "range");
  asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
               :: "r"(taddr), "r"(r[OFF + 0]),"r"(r[OFF + 1]),"r"(r[OFF + 2]),"r"(r[OFF + 3]),"r"(r[OFF + 4]),"r"(r[OFF + 5]),"r"(r[OFF + 6]),"r"(r[OFF + 7]),"r"(r[OFF + 8]),"r"(r[OFF + 9]),"r"(r[OFF + 10]),"r"(r[OFF + 11]),"r"(r[OFF + 12]),"r"(r[OFF + 13]),"r"(r[OFF + 14]),"r"(r[OFF + 15]),"r"(r[OFF + 16]),"r"(r[OFF + 17]),"r"(r[OFF + 18]),"r"(r[OFF + 19]),"r"(r[OFF + 20]),"r"(r[OFF + 21]),"r"(r[OFF + 22]),"r"(r[OFF + 23]),"r"(r[OFF + 24]),"r"(r[OFF + 25]),"r"(r[OFF + 26]),"r"(r[OFF + 27]),"r"(r[OFF + 28]),"r"(r[OFF + 29]),"r"(r[OFF + 30]),"r"(r[OFF + 31])
               : "memory");
}
// 32 lanes x 32 bit store, 16 consecutive columns per thread.
KS_DEV void ks_tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors (tcgen05 shared-memory matrix descriptor, 64 bit):
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) version = 1,
//   [49,52) base offset, [52] LBO mode, [61,64) layout (2 = 128B swizzle).
// ---------------------------------------------------------------------------
KS_DEV uint64_t ks_umma_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3fffu);
  d |= uint64_t((lbo_bytes >> 4) & 0x3fffu) << 16;
  d |= uint64_t((sbo_bytes >> 4) & 0x3fffu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(2) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D:
//   [4,6) D format (1 = f32), [7,10) A format (1 = bf16), [10,13) B format,
//   [15] A major (0 = K), [16] B major (1 = MN), [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t ks_idesc_bf16_f32(int m, int n, bool a_mn_major, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(a_mn_major) << 15) | (uint32_t(b_mn_major) << 16) |
         (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace ks {
int map_cuda(cudaError_t e);          // cudaError_t -> ks_status
int check_arch_sm100();               // KS_ERR_ARCH unless the device is 10.x
int encode_tmap_2d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t inner, uint64_t outer,
                   uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                   CUtensorMapSwizzle swz);
int encode_tmap_3d(CUtensorMap *m, CUtensorMapDataType dt, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                   uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2,
                   CUtensorMapSwizzle swz);
int sm_count();
// Device address of a __device__ variable of this library in the driver
// context current on this thread, resolved once per (context, symbol) with
// cudaGetSymbolAddress and cached.
int symbol_address(const void *symbol, void **out);
// Wait settings for kernels launched on the current device (error word
// address resolved once per device, limit from ks_set_wait_limit_ns).
KsWait wait_ctx();
void set_reason(char *buf, size_t len, const char *fmt, ...);
}  // namespace ks
