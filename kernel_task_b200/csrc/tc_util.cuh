// Shared helpers of the tcgen05 kernels (ring_tc05.cu): UMMA shared-memory
// descriptors and instruction descriptors, single-lane MMA issue and commit, tcgen05 fences,
// bounded mbarrier waits, TMA bulk copies, named barriers and TMEM loads.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "device_util.cuh"

namespace trr {

constexpr unsigned kWaitLimit = 1u << 16;   // try_wait rounds before a wait gives up
constexpr unsigned kSpinLimit = 1u << 26;   // test_wait polls before a spinning wait gives up
constexpr unsigned kSuspendNs = 20000;       // suspend-time hint of one try_wait round

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

// UMMA shared-memory matrix descriptors (sm_100 version field = 1).
__device__ __forceinline__ uint64_t desc_plain(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (uint64_t)((lbo >> 4) & 0x3FFFu) << 16 |
         (uint64_t)((sbo >> 4) & 0x3FFFu) << 32 | (uint64_t)1 << 46;
}
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (uint64_t)1 << 16 | (uint64_t)(1024 >> 4) << 32 |
         (uint64_t)1 << 46 | (uint64_t)2 << 61;
}

// kind::f16 instruction descriptor: A and B both of type E (fp16 or bf16), fp32 D, K-major.
template <typename E>
__host__ __device__ constexpr uint32_t umma_idesc(int M, int N) {
  return (1u << 4) | ((std::is_same<E, __nv_bfloat16>::value ? 1u : 0u) << 7) |
         ((std::is_same<E, __nv_bfloat16>::value ? 1u : 0u) << 10) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// tcgen05.mma, issued by one elected lane of a converged warp: every lane executes the call with
// the same operands, so the descriptor arithmetic stays warp-uniform.
__device__ __forceinline__ void umma_one(uint32_t dtmem, uint64_t da, uint64_t db, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\tsetp.ne.b32 p, %4, 0;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n" ::"r"(
          dtmem),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void commit_one(uint32_t mbar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}\n" ::"r"(
          mbar)
      : "memory");
}


__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t mbar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(mbar), "r"(parity)
      : "memory");
  return done != 0;
}

// One try_wait round: the thread may be suspended until the phase completes or about
// kSuspendNs pass, without spinning on the barrier.
__device__ __forceinline__ bool mbar_try(uint32_t mbar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(done)
      : "r"(mbar), "r"(parity), "r"(kSuspendNs)
      : "memory");
  return done != 0;
}

// Bounded wait for the phase with parity `parity` to complete.  Gives up at once when the CTA's
// abort flag is set, and sets it when the bound runs out.
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity, volatile int* abort) {
  if (mbar_test(mbar, parity)) return true;  // already complete: a test costs a few cycles
  for (unsigned i = 0; i < kWaitLimit; ++i) {
    if (mbar_try(mbar, parity)) return true;
    if (*abort) return false;
  }
  *abort = 1;
  return false;
}


// Spinning bounded wait of one thread (test_wait polls; the abort flag is checked every 256).
// `limit` polls without completion make the wait give up and raise the CTA's abort flag.
#ifndef TRR_SPIN_BACKOFF_NS
#define TRR_SPIN_BACKOFF_NS 0
#endif
#ifndef TRR_SPIN_TRYWAIT
#define TRR_SPIN_TRYWAIT 1000
#endif
__device__ __forceinline__ bool mbar_spin(uint32_t mbar, uint32_t parity, volatile int* abort,
                                          unsigned limit = kSpinLimit) {
  for (unsigned i = 0; !mbar_test(mbar, parity); ++i) {
    if ((i & 255) == 255 && *abort) return false;
    if (i >= limit) {
      *abort = 1;
      return false;
    }
#if TRR_SPIN_TRYWAIT
    if (i >= 4) {
      uint32_t done;
      asm volatile(
          "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
          "selp.u32 %0, 1, 0, p;\n\t}\n"
          : "=r"(done)
          : "r"(mbar), "r"(parity), "r"(TRR_SPIN_TRYWAIT)
          : "memory");
      if (done) return true;
    }
#endif
#if TRR_SPIN_BACKOFF_NS
    if (i >= 4) __nanosleep(TRR_SPIN_BACKOFF_NS);
#endif
  }
  return true;
}

// A converged warp waits together and agrees on the outcome.  It spins on test_wait instead of
// the suspending try_wait: the MMA-issuing warps sit on the critical path of every ring piece,
// and a suspended warp resumed 0.1-0.25 us after the phase completed (measured with globaltimer
// marks; spinning cut the c2 T = 32 call from 57 to 50 us).
__device__ __forceinline__ bool warp_wait(uint32_t mbar, uint32_t parity, volatile int* abort,
                                          unsigned limit = kSpinLimit) {
  return __all_sync(0xffffffffu, mbar_spin(mbar, parity, abort, limit));
}

// Bounded wait that ignores the abort flag: draining the CTA's own work in flight.
__device__ __forceinline__ void mbar_drain(uint32_t mbar, uint32_t parity) {
  if (mbar_test(mbar, parity)) return;
  for (unsigned i = 0; i < kWaitLimit && !mbar_try(mbar, parity); ++i) {
  }
}

// Spinning bounded wait that ignores the abort flag: an issuing warp waits for its own
// tensor-core work on every exit path (it completes on its own, so the bound is never reached
// in practice).
__device__ __forceinline__ void mbar_drain_spin(uint32_t mbar, uint32_t parity) {
  for (unsigned i = 0; i < kSpinLimit && !mbar_test(mbar, parity); ++i) {
  }
}

__device__ __forceinline__ void mbar_arrive(uint32_t mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(mbar) : "memory");
}

// One thread: TMA bulk copy of `bytes` (multiple of 16) global -> shared, completing on `mbar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t mbar) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(mbar), "r"(bytes)
               : "memory");
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(mbar)
      : "memory");
}

// One thread: TMA bulk copy global -> shared completing on `mbar`, without an arrival (the
// caller's one mbarrier.arrive.expect_tx announces the bytes of every copy of the phase).
__device__ __forceinline__ void bulk_copy(uint32_t dst, const void* src, uint32_t bytes,
                                          uint32_t mbar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::
          "r"(dst),
      "l"(src), "r"(bytes), "r"(mbar)
      : "memory");
}

// Named barrier `id` over `n` threads (a multiple of 32): wait for all of them ...
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(n) : "memory");
}
// ... or arrive without waiting (the producer side of a producer -> consumer hand-off).
__device__ __forceinline__ void named_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;\n" ::"r"(id), "r"(n) : "memory");
}

// The two halves of a cluster barrier, so that work between them overlaps its latency: every
// thread's earlier memory accesses are released at cluster scope by the arrive and acquired
// by the wait (both executed by every thread of the CTA, warps converged).
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// Arrival on a device-scope counter: returns the previous value.  Release: called by one thread
// after a CTA barrier, it publishes the writes that every thread of the CTA made before the
// barrier; acquire: the caller (and, after a following CTA barrier, every thread) sees the
// writes that the earlier arrivals published.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], %2;\n"
               : "=r"(old)
               : "l"(p), "r"(v)
               : "memory");
  return old;
}

template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]);
template <>
__device__ __forceinline__ void tmem_ld<8>(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
template <>
__device__ __forceinline__ void tmem_ld<16>(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// Byte offset of element (row r, k) in a K-major matrix with K (a multiple of 8) columns, no
// swizzle: 8-row x 16-byte core matrices, LBO 128 B along K, SBO = K / 8 * 128 B between
// 8-row groups.  The layout every packed tcgen05 operand uses.
__host__ __device__ __forceinline__ uint32_t kmajor_offset(int r, int k, int K) {
  return (uint32_t)((r >> 3) * (K >> 3) * 128 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

}  // namespace trr
