// K3 (prefill / batched form) + K4: sequence-parallel tensor parallelism over NVLink peer memory.
//
// A Megatron layer under TP=W has two row-parallel GEMMs (attention output, FFN down) whose partial
// outputs must be summed over ranks, each followed by an RMSNorm whose result feeds a
// column-parallel GEMM (qkv, gate|up) on every rank.  Here that is, per site:
//
//   row-parallel GEMM, epilogue EPI_RS_PUSH      every finished output tile is stored straight into
//     (gemm_tc.cu)                               the owner rank's receive slots over NVLink and
//                                                flagged there (reduce-scatter fused into the GEMM:
//                                                the transfer of tile i overlaps the math of i+1);
//   sp_reduce_norm_ag_kernel (this file)         the owner waits for the tiles of its rows, adds the
//                                                W partials in rank order into its rows of the
//                                                residual stream, applies RMSNorm and pushes the
//                                                fp16/bf16 rows into every rank's gather buffer with a
//                                                flag per row (the all-gather, issued per row);
//   column-parallel GEMM with an SpWait          its activation producer waits for the row flags of
//     (gemm_tc.cu)                               each token tile before the TMA load, so the first
//                                                tiles start while later rows are still in flight.
//
// The residual stream is sharded by token rows (rank r owns rows [r*chunk, (r+1)*chunk)).  Traffic
// per rank and site: (W-1)/W of T*N*4 bytes out (RS) and (W-1)/W of T*N*2 bytes in (AG), against
// 2*(W-1)/W of T*N*4 for an all-reduce of the f32 partials.  No NCCL call on this path.
//
// Reuse of the buffers without a barrier: a peer writes the slots of row i for the next call only
// after its column-parallel GEMM consumed row i of the gather buffer, which this rank pushed only
// after reading its slots of row i; the same chain protects the gather buffer.  Epochs are per-site
// call counters in device memory, advanced on every rank by the last CTA of this kernel, so every
// rank agrees on them without exchanging them and the whole step is CUDA-graph replayable.  Every
// wait is bounded by %globaltimer; on expiry the error word records 0x500 | (source rank) and the
// kernel still advances the epoch, so the host raises instead of the ranks hanging.
//
// Parity: MultiGpuManager::reduce_scatter / all_gather (backend/src/cuda_multi_gpu.rs:217-233) and
// the column/row-parallel linear layers (:254-328), which are host-side stubs in the reference.
#include "common.cuh"
#include "launch.h"
#include "sysflags.cuh"

namespace barq {

namespace {

constexpr int kRedThreads = 256;

BARQ_DEV float block_sum_256(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kRedThreads / 32; ++i) t += red[i];
  __syncthreads();
  return t;
}

}  // namespace

// grid: one CTA per owned row (at least one CTA, so that a rank with no rows still advances its
// epoch).  256 threads, 4 columns per thread per pass.
__global__ void __launch_bounds__(kRedThreads) sp_reduce_norm_ag_kernel(SpReduceArgs a) {
  __shared__ uint32_t ep_s;
  __shared__ int fail_s;
  __shared__ float red[kRedThreads / 32];
  if (threadIdx.x == 0) {
    ep_s = *a.epoch + 1;
    fail_s = 0;
  }
  __syncthreads();
  const uint32_t ep = ep_s;
  const int row0 = a.rank * a.chunk;
  const int rows = max(0, min(a.T, row0 + a.chunk) - row0);
  const int lr = blockIdx.x;  // local row
  if (lr < rows) {
    const int grow = row0 + lr;  // global token row
    if (a.n_src > 0) {
      // the GEMM tiles covering this row from every source rank: one flag per (source, n tile)
      const int tt = grow / a.gemm_bn;
      for (int i = threadIdx.x; i < a.n_src * a.n_tiles; i += blockDim.x) {
        const int src = i / a.n_tiles, nt = i - src * a.n_tiles;
        const uint32_t* f = a.rs_flags + (size_t)src * a.max_tiles + nt + (size_t)a.n_tiles * tt;
        if (!wait_epoch_sys(f, ep, a.wait_ns)) {
          fail_s = 1;
          atomicExch(a.err, 0x500 | src);
        }
      }
      __syncthreads();
    }
    if (!fail_s) {
      float* xr = a.x + (size_t)lr * a.H;
      float ss = 0.f;
      for (int k = threadIdx.x * 4; k < a.H; k += kRedThreads * 4) {
        float4 v = *reinterpret_cast<float4*>(xr + k);
        for (int src = 0; src < a.n_src; ++src) {  // rank order: the same bits on every rank
          const float4 p = __ldcg(reinterpret_cast<const float4*>(a.slots + ((size_t)src * a.chunk + lr) * a.H + k));
          v.x += p.x;
          v.y += p.y;
          v.z += p.z;
          v.w += p.w;
        }
        if (a.bias) {
          const float4 b = *reinterpret_cast<const float4*>(a.bias + k);
          v.x += b.x;
          v.y += b.y;
          v.z += b.z;
          v.w += b.w;
        }
        if (a.n_src > 0 || a.bias) *reinterpret_cast<float4*>(xr + k) = v;
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      __syncthreads();  // x row written before it is re-read below
      const float rstd = rsqrtf(block_sum_256(ss, red) / (float)a.H + a.eps);
      for (int k = threadIdx.x * 4; k < a.H; k += kRedThreads * 4) {
        const float4 v = *reinterpret_cast<const float4*>(xr + k);
        const float4 w = *reinterpret_cast<const float4*>(a.norm_w + k);
        uint2 pk;
        if (a.out_f16) {
          __half2 lo = __floats2half2_rn(v.x * rstd * w.x, v.y * rstd * w.y);
          __half2 hi = __floats2half2_rn(v.z * rstd * w.z, v.w * rstd * w.w);
          pk = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
        } else {
          __nv_bfloat162 lo = __floats2bfloat162_rn(v.x * rstd * w.x, v.y * rstd * w.y);
          __nv_bfloat162 hi = __floats2bfloat162_rn(v.z * rstd * w.z, v.w * rstd * w.w);
          pk = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
        }
        for (int q = 0; q < a.W; ++q)  // all-gather: this row into every rank's buffer (NVLink stores)
          if (!a.self_only || q == a.rank)
            *reinterpret_cast<uint2*>(static_cast<uint16_t*>(a.ag[q]) + (size_t)grow * a.H + k) = pk;
      }
      __threadfence_system();
    }
    // flagged even after a failed wait (the error word is set): peers then stop waiting at once
    __syncthreads();
    if (threadIdx.x < a.W && (!a.self_only || (int)threadIdx.x == a.rank))
      st_release_sys(a.ag_flags[threadIdx.x] + grow, ep);
  }
  // the last CTA out advances the epoch and clears the arrival counter for the next call
  __syncthreads();
  if (threadIdx.x == 0 && atom_add_acq_rel_gpu(a.done, 1) == (int)gridDim.x - 1) {
    *a.done = 0;
    *a.epoch = ep;
  }
}

__global__ void __launch_bounds__(256) sp_ag_wait_kernel(const uint32_t* flags, const uint32_t* epoch, int T,
                                                         int* err, unsigned long long wait_ns) {
  const uint32_t ep = *epoch;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < T; r += gridDim.x * blockDim.x)
    if (!wait_epoch_sys(flags + r, ep, wait_ns)) atomicExch(err, 0x600);
}

int sp_reduce_norm_ag(const SpReduceArgs& a, cudaStream_t st) {
  if (a.W < 1 || a.W > kSpMaxRanks || a.rank < 0 || a.rank >= a.W || a.chunk * a.W < a.T) return -1;
  if (a.H % 4 || (reinterpret_cast<uintptr_t>(a.x) & 15) || (a.slots && (reinterpret_cast<uintptr_t>(a.slots) & 15)))
    return -2;
  if (a.n_src > 0 && (!a.rs_flags || a.gemm_bn <= 0 || a.n_tiles <= 0)) return -3;
  for (int q = 0; q < a.W; ++q)
    if (!a.ag[q] || !a.ag_flags[q] || (reinterpret_cast<uintptr_t>(a.ag[q]) & 7)) return -4;
  const int row0 = a.rank * a.chunk;
  const int rows = max(0, min(a.T, row0 + a.chunk) - row0);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows > 0 ? rows : 1);
  cfg.blockDim = dim3(kRedThreads);
  cfg.stream = st;
  return cudaLaunchKernelEx(&cfg, sp_reduce_norm_ag_kernel, a) == cudaSuccess ? 0 : -20;
}

int sp_ag_wait(const uint32_t* flags, const uint32_t* epoch, int T, int* err, unsigned long long wait_ns,
               cudaStream_t st) {
  if (T <= 0) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((T + 255) / 256);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  return cudaLaunchKernelEx(&cfg, sp_ag_wait_kernel, flags, epoch, T, err, wait_ns) == cudaSuccess ? 0 : -20;
}

}  // namespace barq
