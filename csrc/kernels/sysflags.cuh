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
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
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

// Spin until the 64-bit word at p carries epoch ep in its high half (value in the low half), giving
// up after wait_ns of %globaltimer or once another thread has recorded a peer timeout in *err.
__device__ __forceinline__ bool wait_pair_sys(const uint64_t* p, uint32_t ep, uint64_t wait_ns, const int* err,
                                              uint64_t& out) {
  const uint64_t t0 = gtimer();
  for (uint32_t i = 0;; ++i) {
    const uint64_t v = ld_relaxed_sys_u64(p);
    if ((uint32_t)(v >> 32) == ep) {
      out = v;
      return true;
    }
    if ((i & 255) == 255) {
      if (gtimer() - t0 > wait_ns) return false;
      if (err && (*(const volatile int*)err & 0xF00) == 0x300) return false;
    }
  }
}

}  // namespace barq
