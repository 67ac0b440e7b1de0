// Blackwell (sm_100a) building blocks in inline PTX: mbarriers with bounded waits, TMA tile loads,
// tcgen05 TMEM allocation / MMA / commit / load, and UMMA shared-memory descriptors.
//
// Every TMA copy here reads this GPU's own memory into the issuing CTA only.
#pragma once
#include <cuda.h>
#include <stdint.h>
#include "common.cuh"

namespace barq {
namespace tc {

BARQ_DEV uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

BARQ_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}
BARQ_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
BARQ_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
BARQ_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
BARQ_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

BARQ_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: polls a hardware-suspended try_wait until the phase flips, another role reported
// an error, or ~2 s of %globaltimer elapsed; on expiry the error word is set (0x100 | call site)
// and false is returned so every role can unwind and the kernel returns normally.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
BARQ_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait ignoring the error word (used to drain copies in flight before a CTA exits); bounded.
BARQ_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 0;; ++i) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((i & 255) == 255 && globaltimer_ns() - t0 > kWaitLimitNs) return false;
  }
}
BARQ_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* err, int site) {
  if (mbar_test_wait(bar, parity)) return true;  // non-blocking probe: cheaper when already complete
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*err) return false;
    if ((i & 255) == 0 && globaltimer_ns() - t0 > kWaitLimitNs) break;
  }
  *err = 0x100 | site;
  return false;
}

BARQ_DEV void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2D tiled TMA load of box (x, y) into shared memory, completion on `bar` (transaction bytes).
BARQ_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
      : "memory");
}
BARQ_DEV void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---- TMEM
BARQ_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols));
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
BARQ_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
BARQ_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
BARQ_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, f32 accumulate), cta_group::1.
BARQ_DEV void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16: A's 128 rows are TMEM lanes, its K elements
// packed two per 32-bit column (even k in the low half).
BARQ_DEV void mma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// 32 lanes x 8 consecutive 32-bit columns from registers into TMEM (warp w: lanes 32*(w%4) .. +31).
BARQ_DEV void tmem_st8(uint32_t taddr, uint4 lo, uint4 hi) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(lo.x),
               "r"(lo.y), "r"(lo.z), "r"(lo.w), "r"(hi.x), "r"(hi.y), "r"(hi.z), "r"(hi.w)
               : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns from registers into TMEM.
BARQ_DEV void tmem_st16(uint32_t taddr, const uint4* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0].x), "r"(v[0].y), "r"(v[0].z), "r"(v[0].w), "r"(v[1].x), "r"(v[1].y), "r"(v[1].z), "r"(v[1].w),
      "r"(v[2].x), "r"(v[2].y), "r"(v[2].z), "r"(v[2].w), "r"(v[3].x), "r"(v[3].y), "r"(v[3].z), "r"(v[3].w)
      : "memory");
}
BARQ_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrive on `bar` once every previously issued tcgen05.mma of this thread has completed.
BARQ_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}

// 32 lanes x 32 columns of f32 from TMEM (warp w may only touch lanes 32*(w%4) .. +31).
BARQ_DEV void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,"
      "%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// UMMA shared-memory descriptor, K-major operand in the 128-byte swizzle canonical layout:
// rows of 64 bf16 (128 B), 8-row groups 1024 B apart (SBO), 16-byte chunk c of row r stored at
// chunk position c ^ (r % 8).  Tile base must be 1024-byte aligned.
BARQ_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);       // start address
  d |= (uint64_t)1 << 16;                        // LBO (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;              // SBO
  d |= (uint64_t)1 << 46;                        // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                        // SWIZZLE_128B
  return d;
}

// UMMA shared-memory descriptor, MN-major operand in the 128-byte swizzle canonical layout: along
// MN, 64 consecutive 16-bit elements fill one 128-byte row; rows are consecutive K indices, 8-row
// groups 1024 B apart (SBO); the next 64 MN elements start `lbo` bytes further (LBO).  This is
// the layout a 2D TMA box {64, rows} with SWIZZLE_128B writes when its inner dimension is MN
// (e.g. V tiles [keys][D] used as the B operand of P V).  Tile base must be 1024-byte aligned.
BARQ_DEV uint64_t umma_desc_sw128_mn(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);       // start address
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;   // LBO: stride between 64-element MN blocks
  d |= (uint64_t)(1024 >> 4) << 32;              // SBO: stride between 8-row K groups
  d |= (uint64_t)1 << 46;                        // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                        // SWIZZLE_128B
  return d;
}
// Instruction-descriptor bit selecting an MN-major B operand (bit 16; 0 = K-major).
constexpr uint32_t kIdescBMajorMN = 1u << 16;

// Instruction descriptor for kind::f16 with bf16 A/B, f32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4)            // D format f32
         | (1u << 7)          // A bf16
         | (1u << 10)         // B bf16
         | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor for kind::f16 with f16 A/B, f32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

}  // namespace tc
}  // namespace barq
