// K3 (decode form): one-shot all-reduce over NVLink peer memory, fused with the residual add.
//
// Row-parallel layers (attention output, FFN down) leave a partial sum on every rank.  Each rank's
// GEMV/GEMM writes its partial into its own buffer of a symmetric allocation (every rank maps every
// peer's buffer); this kernel then, on every rank,
//   1. (per block) signals "partial ready" to each peer: a release store of its epoch into the
//      peer's flag slot [block][my rank], and waits until every peer's flag in its own slots reached
//      the same epoch (acquire loads, bounded by a wait limit measured on %globaltimer -- long
//      enough to absorb host-side skew between ranks such as CUDA-graph capture; on expiry the error
//      word is set and the block skips the sum but still advances its epoch, keeping ranks aligned);
//   2. reads the partials of all ranks straight from peer memory (plain per-thread loads over
//      NVLink, no TMA) and adds their sum into the local residual stream x.
// Epochs live in device memory (one counter per block, advanced by the kernel), so the kernel is
// CUDA-graph replayable.  Two partial buffers alternate between the two all-reduces of a layer: a
// rank rewrites a buffer only after the next all-reduce's barrier, which every peer passes only
// after its previous kernels (the reads of that buffer) have completed.
//
// Parity: MultiGpuManager::all_reduce / NcclCommunicator::all_reduce_sum
// (backend/src/cuda_multi_gpu.rs:207-213, 431-436), which return Unsupported in the reference.
#include "common.cuh"
#include "launch.h"
#include "pdl.cuh"
#include "sysflags.cuh"

namespace barq {

__global__ void __launch_bounds__(256) allreduce_add_kernel(ArArgs a) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  __shared__ uint32_t ep_s;
  __shared__ int fail_s;
  if (threadIdx.x == 0) {
    ep_s = a.epoch[b] + 1;
    fail_s = 0;
  }
  __syncthreads();
  const uint32_t ep = ep_s;
  if (threadIdx.x < a.world) {
    const int peer = threadIdx.x;
    __threadfence_system();  // this rank's partial (written by the previous kernel) before the flag
    if (!a.skip_signal) st_release_sys(a.flags[peer] + b * kArMaxRanks + a.rank, ep);
    const uint32_t* mine = a.flags[a.rank] + b * kArMaxRanks + peer;
    const uint64_t t0 = gtimer();
    for (uint32_t i = 0;; ++i) {
      if ((int)(ld_acquire_sys(mine) - ep) >= 0) break;
      if ((i & 1023) == 1023 && gtimer() - t0 > a.wait_ns) {
        fail_s = 1;
        atomicExch(a.err, 0x300 | peer);
        break;
      }
    }
  }
  __syncthreads();
  if (fail_s) {  // a peer never arrived: x is left unchanged, the host raises on the error word
    if (threadIdx.x == 0) a.epoch[b] = ep;
    return;
  }
  // x[i] += sum_r partial_r[i] over this block's grid-stride share, float4 at a time
  // every rank's float4 is loaded before any is added (all peers' NVLink reads in flight at once),
  // then summed in rank order
  const int n4 = a.n / 4;
  for (int i = b * blockDim.x + threadIdx.x; i < n4; i += gridDim.x * blockDim.x) {
    float4 v[kArMaxRanks];
#pragma unroll
    for (int r = 0; r < kArMaxRanks; ++r)
      v[r] = r < a.world ? __ldcg(reinterpret_cast<const float4*>(a.bufs[r]) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 acc = reinterpret_cast<float4*>(a.x)[i];
#pragma unroll
    for (int r = 0; r < kArMaxRanks; ++r) {
      if (r >= a.world) break;
      acc.x += v[r].x;
      acc.y += v[r].y;
      acc.z += v[r].z;
      acc.w += v[r].w;
    }
    reinterpret_cast<float4*>(a.x)[i] = acc;
  }
  for (int i = n4 * 4 + b * blockDim.x + threadIdx.x; i < a.n; i += gridDim.x * blockDim.x) {
    float acc = a.x[i];
    for (int r = 0; r < a.world; ++r) acc += a.bufs[r][i];
    a.x[i] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) a.epoch[b] = ep;
}

// ---- NVLS form (two-shot through NVSwitch multicast): `a.mc` is the multicast address of this
// call's partial buffer (the same offset in every rank's symmetric allocation).
//   1. barrier (as above): every rank's partial is in place;
//   2. rank r reduces its slice [r S, (r + 1) S) of the float4 range with
//      multimem.ld_reduce.add (the switch sums the W partials) and writes the sum back to every
//      rank's buffer with multimem.st (slices are disjoint, so the write-back is in place);
//   3. second barrier: every rank's stores have landed;
//   4. x += the local buffer (now the full sum).
// Each GPU pulls n / W reduced values and pushes n / W, against (W - 1) n pulled by the one-shot
// form, and all ranks add bit-identical sums (one reduction per element, done once), which keeps
// tensor-parallel replicas of the residual stream identical.  The n % 4 tail is summed from peer
// memory in rank order.  Opt-in (BARQ_AR_MULTIMEM=1) until it has run on NVSwitch GPUs.
__device__ __forceinline__ float4 multimem_ld_reduce_add_v4(const float* mc) {
  float4 v;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(mc)
               : "memory");
  return v;
}
__device__ __forceinline__ void multimem_st_v4(float* mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}

// Per-block barrier with every peer at epoch `ep` (threads < world signal and wait); false when a
// peer did not arrive within the wait limit (the error word names it).
__device__ __forceinline__ bool ar_block_barrier(const ArArgs& a, int b, uint32_t ep, int* fail_s) {
  if (threadIdx.x < a.world) {
    const int peer = threadIdx.x;
    __threadfence_system();  // this rank's stores (partial, or multicast write-back) before the flag
    if (!a.skip_signal) st_release_sys(a.flags[peer] + b * kArMaxRanks + a.rank, ep);
    const uint32_t* mine = a.flags[a.rank] + b * kArMaxRanks + peer;
    const uint64_t t0 = gtimer();
    for (uint32_t i = 0;; ++i) {
      if ((int)(ld_acquire_sys(mine) - ep) >= 0) break;
      if ((i & 1023) == 1023 && gtimer() - t0 > a.wait_ns) {
        *fail_s = 1;
        atomicExch(a.err, 0x300 | peer);
        break;
      }
    }
  }
  __syncthreads();
  return !*fail_s;
}

__global__ void __launch_bounds__(256) allreduce_add_mc_kernel(ArArgs a) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.x;
  __shared__ uint32_t ep_s;
  __shared__ int fail_s;
  if (threadIdx.x == 0) {
    ep_s = a.epoch[b];
    fail_s = 0;
  }
  __syncthreads();
  const uint32_t ep = ep_s;
  const int n4 = a.n / 4;
  const int S = (n4 + a.world - 1) / a.world;  // float4 slice per rank
  const int lo = min(n4, a.rank * S), hi = min(n4, lo + S);
  const int stride = gridDim.x * blockDim.x;
  float* local = const_cast<float*>(a.bufs[a.rank]);
  bool ok = ar_block_barrier(a, b, ep + 1, &fail_s);
  // the partials were written through unicast addresses and are read here through the multicast
  // alias (and the sums written back through it are read below through the unicast one)
  asm volatile("fence.proxy.alias;" ::: "memory");
  if (ok) {
    for (int i = lo + b * blockDim.x + threadIdx.x; i < hi; i += stride)
      multimem_st_v4(a.mc + 4 * (size_t)i, multimem_ld_reduce_add_v4(a.mc + 4 * (size_t)i));
    __syncthreads();
    ok = ar_block_barrier(a, b, ep + 2, &fail_s);
  }
  asm volatile("fence.proxy.alias;" ::: "memory");
  if (ok) {
    // this block's share of every rank's slice: the same (slice offset, thread) positions as step 2
    for (int r = 0; r < a.world; ++r) {
      const int rlo = min(n4, r * S), rhi = min(n4, rlo + S);
      for (int i = rlo + b * blockDim.x + threadIdx.x; i < rhi; i += stride) {
        const float4 s = __ldcv(reinterpret_cast<const float4*>(local) + i);
        float4 acc = reinterpret_cast<float4*>(a.x)[i];
        acc.x += s.x;
        acc.y += s.y;
        acc.z += s.z;
        acc.w += s.w;
        reinterpret_cast<float4*>(a.x)[i] = acc;
      }
    }
    if (b == 0)
      for (int i = n4 * 4 + threadIdx.x; i < a.n; i += blockDim.x) {
        float acc = a.x[i];
        for (int r = 0; r < a.world; ++r) acc += a.bufs[r][i];
        a.x[i] = acc;
      }
  }
  __syncthreads();
  if (threadIdx.x == 0) a.epoch[b] = ep + 2;  // both barriers' epochs are used, also after a timeout
}

int allreduce_add(const ArArgs& a, cudaStream_t st) {
  if (a.world < 1 || a.world > kArMaxRanks || a.rank < 0 || a.rank >= a.world) return -1;
  if (a.blocks < 1 || a.blocks > kArMaxBlocks) return -2;
  if (reinterpret_cast<uintptr_t>(a.x) & 15) return -3;
  for (int r = 0; r < a.world; ++r)
    if (reinterpret_cast<uintptr_t>(a.bufs[r]) & 15) return -3;
  if (a.mc && (reinterpret_cast<uintptr_t>(a.mc) & 15)) return -3;
  if (a.n <= 0) return 0;
  auto kern = a.mc ? allreduce_add_mc_kernel : allreduce_add_kernel;
  return launch_pdl(kern, dim3(a.blocks), dim3(256), 0, st, a) == cudaSuccess ? 0 : -20;
}

}  // namespace barq
