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

int allreduce_add(const ArArgs& a, cudaStream_t st) {
  if (a.world < 1 || a.world > kArMaxRanks || a.rank < 0 || a.rank >= a.world) return -1;
  if (a.blocks < 1 || a.blocks > kArMaxBlocks) return -2;
  if (reinterpret_cast<uintptr_t>(a.x) & 15) return -3;
  for (int r = 0; r < a.world; ++r)
    if (reinterpret_cast<uintptr_t>(a.bufs[r]) & 15) return -3;
  if (a.n <= 0) return 0;
  return launch_pdl(allreduce_add_kernel, dim3(a.blocks), dim3(256), 0, st, a) == cudaSuccess ? 0 : -20;
}

}  // namespace barq
