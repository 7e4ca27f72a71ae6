// rfsn_common.cuh — device helpers shared by the RFSN B200 kernels.
//
// * 1-D bulk TMA copies (cp.async.bulk global -> shared, completion counted on
//   an mbarrier) with explicit 16-byte alignment handling.
// * mbarrier wrappers whose waits are bounded by %globaltimer: a wait that
//   does not complete within kWaitLimitNs returns false so the kernel can set
//   an error status and leave instead of hanging the GPU.
// * fp16 <-> fp32 helpers operating on raw uint16 bit patterns.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/rfsn_b200.h"

namespace rfsn {

// A bounded device wait gives up after this many nanoseconds (1 s).
constexpr uint64_t kWaitLimitNs = 1000ull * 1000ull * 1000ull;

// Device status codes written to rfsn_attn_args::device_status.
constexpr int kDevStatusTimeoutFull = 1;
constexpr int kDevStatusTimeoutEmpty = 2;
constexpr int kDevStatusBadSegment = 3;
constexpr int kDevStatusTicket = 4;
constexpr int kDevStatusPeerTimeout = 5;  // a peer rank's gather signal did not arrive in time

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
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

// Bounded wait for the phase with the given parity.  Returns false on timeout
// or when *abort becomes non-zero (another thread already timed out).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 15u) == 0) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) return false;
    }
  }
}

// 1-D bulk copy global -> shared::cta (a non-cluster CTA is its own cluster),
// completion reported as transaction bytes on `bar`.  dst, src and bytes must
// be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

constexpr unsigned long long kTagMask = (1ull << 48) - 1ull;

// Count one arrival on ticket *t for the launch tagged `tag` (a launch counter the kernel
// keeps in its workspace); returns 1 if it was arrival number `target` of this launch, 0 if
// not, -1 if the ticket could not be taken.  A ticket holding another launch's tag counts as
// zero.  Each failed swap means another CTA's succeeded, and at most 0xffff CTAs arrive on
// one ticket, so the loop bound is never reached in a healthy launch.
__device__ __forceinline__ int take_ticket(unsigned long long* t, unsigned long long tag, int target) {
  unsigned long long cur = *reinterpret_cast<volatile unsigned long long*>(t);
  for (int it = 0; it < 0x10000 + 16; ++it) {
    const unsigned long long nxt = ((cur >> 16) == tag) ? cur + 1ull : ((tag << 16) | 1ull);
    const unsigned long long prev = atomicCAS(t, cur, nxt);
    if (prev == cur) return (int)(nxt & 0xffffull) == target ? 1 : 0;
    cur = prev;
  }
  return -1;
}

// Programmatic dependent launch.  griddep_wait: this thread waits until the grids this launch
// depends on have completed and their memory is visible (a no-op for a launch without that
// dependency).  griddep_launch: this CTA lets dependent launches be scheduled early; they still
// wait in griddep_wait before touching memory this grid writes.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Named barrier among the first `threads` threads of the CTA (id != 0).
__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__host__ __device__ constexpr int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

}  // namespace rfsn
