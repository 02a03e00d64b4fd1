// Inline-PTX helpers for sm_100a: mbarriers, bulk (TMA) copies, fences and
// the bounded waits every kernel uses (a wait that gives up records a
// device error bit instead of spinning forever).
#pragma once

#include <stdint.h>

namespace gdn2 {

// Device error bits, read and cleared by gdn2_read_device_errors().
enum : unsigned {
  DEVERR_MBAR_TIMEOUT = 1u,  // a bounded mbarrier wait gave up
};
// One copy per translation unit (no relocatable device code); each unit
// that launches kernels exposes a host reader (see gdn2_read_device_errors).
static __device__ unsigned g_device_errors = 0;

#define GDN2_DEVICE_ERROR_READER(fn)                                   \
  unsigned fn() {                                                      \
    unsigned v = 0, z = 0;                                             \
    if (cudaMemcpyFromSymbol(&v, g_device_errors, sizeof(v)) != cudaSuccess) return 0; \
    cudaMemcpyToSymbol(g_device_errors, &z, sizeof(z));                \
    return v;                                                          \
  }

// Iterations of try_wait (each suspends for a hardware-chosen time slice)
// before a wait is declared lost: about a second on B200.
constexpr unsigned MBAR_SPIN_LIMIT = 1u << 24;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// this thread's global stores ordered before later bulk (async-proxy) reads of the same bytes
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
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

// Bounded wait for phase `parity` of `bar`.  Returns false (and records
// DEVERR_MBAR_TIMEOUT) if the phase did not complete within `limit`
// try_wait rounds.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity, unsigned limit = MBAR_SPIN_LIMIT) {
  for (unsigned i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicOr(&g_device_errors, DEVERR_MBAR_TIMEOUT);
  return false;
}

// Shared-memory address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
// Bounded wait with cluster-scope acquire (the arrivals come from the peer CTA).
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, unsigned parity) {
  for (unsigned i = 0; i < MBAR_SPIN_LIMIT; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  atomicOr(&g_device_errors, DEVERR_MBAR_TIMEOUT);
  return false;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Pairs of f32 in one 64-bit register for the packed sm_100 multiply / fma
// (mul.rn.f32x2, fma.rn.f32x2: two IEEE round-to-nearest results per
// instruction, the same values as two scalar instructions).
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 f2pk(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2un(f32x2 r, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(r));
}
__device__ __forceinline__ f32x2 f2mul(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f32x2 f2fma(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes).
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* sdst, const void* gsrc, unsigned bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(sdst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// The same copy with an L2 eviction policy for the read lines (l2_policy_*, below).
__device__ __forceinline__ void bulk_g2s_hint(void* sdst, const void* gsrc, unsigned bytes, uint64_t* bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
          "r"(smem_u32(sdst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}

// Bulk prefetch of [gsrc, gsrc + bytes) into L2 (no completion tracking);
// 16-byte aligned address, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* gsrc, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(gsrc), "r"(bytes) : "memory");
}

// 1-D bulk copy shared -> global in the thread's bulk async-group; both
// addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_s2g(void* gdst, const void* ssrc, unsigned bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_u32(ssrc)),
               "r"(bytes)
               : "memory");
}
// The same copy with an L2 eviction policy for the written lines (l2_policy_*).
__device__ __forceinline__ void bulk_s2g_hint(void* gdst, const void* ssrc, unsigned bytes, uint64_t pol) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group.L2::cache_hint [%0], [%1], %2, %3;" ::"l"(gdst),
               "r"(smem_u32(ssrc)), "r"(bytes), "l"(pol)
               : "memory");
}
// Drop the 128-byte L2 line at `p` (128-byte aligned) without writing it back: for scratch whose contents are
// dead (read back already, rewritten before the next read).
__device__ __forceinline__ void discard_l2_line(const void* p) {
  asm volatile("discard.global.L2 [%0], 128;" ::"l"(p) : "memory");
}
// L2 eviction policies for the .L2::cache_hint forms.  Lines that are written or read once and not touched
// again soon (the chunk records, inputs read by one CTA) are marked evict-first, so that L2 keeps the lines
// that are re-read soon (rows prefetched for the next chunk, per-CTA scratch).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// until every bulk copy this thread committed has read its shared-memory source
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Ampere-style per-thread async copy, 16 bytes, L2 only (.cg).
__device__ __forceinline__ void cp_async16(void* sdst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
// the same, 8 bytes, through L1 (.ca: the 8-byte form)
__device__ __forceinline__ void cp_async8(void* sdst, const void* gsrc) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(sdst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace gdn2
