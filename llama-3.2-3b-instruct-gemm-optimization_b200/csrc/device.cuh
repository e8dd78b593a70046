// device.cuh -- sm_100a PTX helpers: mbarriers, 1-D bulk TMA copies, L2 cache
// policies, programmatic dependent launch, E4M3 conversion and the
// m16n8k16 f16 tensor-core MMA.  Every spin-wait here is bounded.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace b2g {

// Device error codes written to the library's error word.
enum : int {
  kErrNone = 0,
  kErrFullWait = 1,   // a consumer waited too long for a TMA stage
  kErrEmptyWait = 2,  // the producer waited too long for consumers
  kErrDrainWait = 3,  // an in-flight copy did not land while aborting
  kErrPeerWait = 4,   // a wait on another GPU's flag expired
  kErrGridWait = 5,   // a grid-wide barrier of the stack kernel expired
};

// A wait gives up after this many nanoseconds of %globaltimer.  Long enough
// that time-slicing with other contexts on a shared GPU cannot trip it.
constexpr unsigned long long kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

// One bounded try: the thread may sleep (up to ~0.1 ms) until the phase completes.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(100000u)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false if
// the budget ran out (the caller records the error and unwinds).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > kWaitBudgetNs) return false;
  }
}

// ---------------------------------------------------------------------------
// 1-D bulk copy global -> shared (TMA), completion counted on an mbarrier.
// src/dst 16-byte aligned, bytes a multiple of 16; this CTA's shared memory only.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

// Bulk prefetch of global memory into L2 (no destination, no completion).
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 16-byte streaming load: read-only path, no L1 allocation, L2 policy hint.
__device__ __forceinline__ uint4 ldg_stream(const void* p, uint64_t policy) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(policy));
  return v;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// ---------------------------------------------------------------------------
// Memory ordering
// ---------------------------------------------------------------------------
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
// Orders this thread's generic-proxy accesses before its later async-proxy
// (TMA) accesses to global memory.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Named barrier over the consumer warps only.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void named_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ---------------------------------------------------------------------------
// Number formats
// ---------------------------------------------------------------------------
// Two E4M3 codes (low byte first) -> f16x2 (low half first); exact.  The
// hardware conversion measured 2.2x the throughput of a shift/mask sequence.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t v16) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((uint16_t)v16));
  return r;
}

// Four E4M3 codes (byte i = element i) -> two f16x2 (elements 0,1 and 2,3).
// The 32-bit word is split into its 16-bit halves in registers (no shift).
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t w, uint32_t& lo, uint32_t& hi) {
  asm("{\n\t.reg .b16 a, b;\n\t"
      "mov.b32 {a, b}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, a;\n\t"
      "cvt.rn.f16x2.e4m3x2 %1, b;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(w));
}

// Atomic add at GPU scope with acquire-release semantics: publishes this
// thread's earlier writes (and those ordered before it) and, for the thread
// that observes the final count, makes the other publishers' writes visible.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

// Arrival on another GPU's counter, relaxed: the caller orders its earlier
// stores with one fence.acq_rel.sys before its arrivals (a release form of
// each arrival would repeat that system-scope fence per peer).
__device__ __forceinline__ void red_relaxed_sys_add(unsigned* p, unsigned v) {
  asm volatile("red.relaxed.sys.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

// Single-copy-atomic 8-byte words at system scope: the flag-in-data exchange
// (a 32-bit round number beside 32 bits of payload in one aligned word) needs
// no fence, since a reader that sees the round sees the payload with it.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// 4 bytes global -> shared without holding a register (completes with
// cp_async_wait_all in the issuing thread).
__device__ __forceinline__ void cp_async4(void* smem_dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\ncp.async.commit_group;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// 16 bytes global -> shared through L2 only (the source may have been
// written by another SM since this one last read it); both addresses
// 16-byte aligned.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))),
               "l"(src)
               : "memory");
}

// float -> E4M3 code, round to nearest even, saturate to +-448.
__device__ __forceinline__ uint8_t f32_to_e4m3(float f) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %1;" : "=h"(r) : "f"(f));
  return static_cast<uint8_t>(r & 0xFF);
}

// half -> E4M3 code, round to nearest even, saturate to +-448.
__device__ __forceinline__ uint8_t f16_to_e4m3(__half h) {
  uint16_t r;
  const uint16_t hb = __half_as_ushort(h);
  const uint32_t pair = (static_cast<uint32_t>(hb) << 16) | hb;
  asm("cvt.rn.satfinite.e4m3x2.f16x2 %0, %1;" : "=h"(r) : "r"(pair));
  return static_cast<uint8_t>(r & 0xFF);
}

// ---------------------------------------------------------------------------
// Tensor-core tile: D(16x8, f32) += A(16x16, f16, row) * B(16x8, f16, col)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(smem_addr(p)));
  return v;
}

// Loads at a 32-bit shared-memory address.
__device__ __forceinline__ uint4 lds128_at(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}

__device__ __forceinline__ uint2 lds64_at(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}

__device__ __forceinline__ uint32_t lds32(const void* p) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)));
  return v;
}

__device__ __forceinline__ void sts128(void* p, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(smem_addr(p)), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ uint2 lds64(const void* p) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_addr(p)));
  return v;
}

}  // namespace b2g
