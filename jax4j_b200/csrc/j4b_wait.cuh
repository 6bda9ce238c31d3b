// Time-bounded waits for device code. Every spin on an mbarrier gives up after kWaitNs of
// %globaltimer (far above any legitimate wait in these kernels), so a barrier that never
// completes ends the kernel with an error status instead of holding the GPU.
#pragma once

#include <cstdint>

namespace j4b {

constexpr uint64_t kWaitNs = 200ull * 1000 * 1000;  // 0.2 s

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// try_wait on the phase with the given parity of the mbarrier at shared address `bar`
__device__ __forceinline__ bool mbar_try_wait_parity(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_wait_timed(uint32_t bar, uint32_t parity) {
  if (mbar_try_wait_parity(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (;;) {
    if (mbar_try_wait_parity(bar, parity)) return true;
    if (global_ns() - t0 > kWaitNs) return false;
  }
}

}  // namespace j4b
