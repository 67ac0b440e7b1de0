// System-scope flag primitives for cross-GPU signalling over NVLink peer memory.
#pragma once
#include <cstdint>

namespace barq {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Spin until *p reaches epoch ep (wrap-safe), giving up after wait_ns of %globaltimer.
__device__ __forceinline__ bool wait_epoch_sys(const uint32_t* p, uint32_t ep, uint64_t wait_ns) {
  const uint64_t t0 = gtimer();
  for (uint32_t i = 0;; ++i) {
    if ((int)(ld_acquire_sys(p) - ep) >= 0) return true;
    if ((i & 1023) == 1023 && gtimer() - t0 > wait_ns) return false;
  }
}

}  // namespace barq
