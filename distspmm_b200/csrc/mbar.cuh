// mbar.cuh — shared-memory mbarrier helpers with bounded waits (sm_90+ PTX).
//
// Every wait gives up after a clock64 budget (about 2 s at B200 clocks by default): it
// records `code` in *err and returns false, so a kernel never spins forever on a copy that
// does not land; the host reads the error word after the launch.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace dsp {

constexpr long long kMbarWaitCycles = 4000000000ll;  // ~2 s at B200 clocks

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(mbar), "r"(count) : "memory");
}

// make initialised barriers visible to the async (TMA) proxy
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive(uint32_t mbar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(mbar) : "memory");
}

// arrive and announce `bytes` of asynchronous copies that complete on this barrier
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t mbar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(mbar),
               "r"(bytes)
               : "memory");
}

// Bounded wait for phase `parity` of an mbarrier; false (and *err = code) after `budget`
// clock64 cycles.
__device__ __forceinline__ bool mbar_wait(uint32_t mbar, uint32_t parity, int *err, int code,
                                          long long budget = kMbarWaitCycles) {
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(mbar), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > budget) {
      if (err) atomicExch(err, code);
      return false;
    }
  }
}

// As mbar_wait, with a suspend-time hint: a thread whose phase is not complete may sleep up
// to hint_ns nanoseconds inside try_wait (woken when the phase completes) instead of
// returning at once, so waiting warps leave the issue slots to working ones.
__device__ __forceinline__ bool mbar_wait_hint(uint32_t mbar, uint32_t parity, uint32_t hint_ns, int *err, int code,
                                               long long budget = kMbarWaitCycles) {
  if (hint_ns == 0) return mbar_wait(mbar, parity, err, code, budget);
  const long long t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(mbar), "r"(parity), "r"(hint_ns)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > budget) {
      if (err) atomicExch(err, code);
      return false;
    }
  }
}

}  // namespace dsp
