// K5 (single-GPU part): MoE routing and dispatch.  The expert GEMMs are the grouped mode of the
// tcgen05 GEMM (gemm_tc.cu) and the combine is that GEMM's EPI_MOE_COMBINE epilogue.
//
// Parity: the reference routes on the CPU (models/src/moe_fused.rs:95-193 top-k + SER,
// models/src/deepseek.rs:140-163 DeepSeek routing) and runs each expert as a separate matmul;
// here routing, the token permutation and the weighted combine stay on the device, so a MoE layer is
// three small kernels plus two grouped GEMMs and needs no device->host copy (CUDA-graph friendly).
//
//   moe_route_kernel     one warp per token: gate (softmax | sigmoid) over E logits, optional
//                        group-limited selection (keep the best topk_group of n_group groups), top-k,
//                        renormalization, SER drop (weights below a threshold, the top expert is
//                        always kept), scale; per-expert counts with atomics.
//   moe_scan_kernel      one block: counts -> row offsets [E+1], cursors, counts cleared.
//   moe_dispatch_kernel  one block per (token, slot): claims a row of its expert and copies the
//                        token's activation row there; records (token, weight) for the combine.
//   moe_combine_kernel   K7: the down GEMM stores weight * y per sorted row; each token then adds
//                        its rows in slot order into the residual stream.  The fixed order keeps the
//                        sum deterministic (no floating-point atomics), whatever order the rows
//                        were claimed in.
#include "common.cuh"
#include "launch.h"
#include "pdl.cuh"
#include "sysflags.cuh"

namespace barq {

constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 8;

// Router logits: out[t, e] = x[t, :] . W[e, :] (x fp16 / bf16 rows, W f32 [E, H], f32 accumulate
// in a fixed order).  A CTA stages kRtTok token rows in shared memory and its 8 warps take experts
// blockIdx.y * kRtExp + warp, + 8, ...; every lane reads W four floats at a time, so each router row
// is read once per CTA and applied to all staged tokens.
constexpr int kRtTok = 8, kRtExp = 32;
template <typename T>
__global__ void __launch_bounds__(256) moe_router_kernel(const T* __restrict__ x, int ldx, const float* __restrict__ w,
                                                          float* __restrict__ out, int Ttot, int E, int H) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) uint8_t rt_smem[];
  T* xs = reinterpret_cast<T*>(rt_smem);  // [kRtTok][H]
  const int t0 = blockIdx.x * kRtTok;
  const int nt = min(kRtTok, Ttot - t0);
  for (int i = threadIdx.x; i < kRtTok * H; i += blockDim.x) {
    const int r = i / H, c = i % H;
    xs[i] = r < nt ? x[(size_t)(t0 + r) * ldx + c] : from_f<T>(0.f);
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e_end = min(E, (int)(blockIdx.y + 1) * kRtExp);
  for (int e = blockIdx.y * kRtExp + warp; e < e_end; e += 8) {
    const float* wr = w + (size_t)e * H;
    float acc[kRtTok];
#pragma unroll
    for (int r = 0; r < kRtTok; ++r) acc[r] = 0.f;
    for (int c = lane * 4; c < H; c += 128) {
      const float4 wv = *reinterpret_cast<const float4*>(wr + c);
#pragma unroll
      for (int r = 0; r < kRtTok; ++r) {
        const T* xr = xs + r * H + c;
        acc[r] = fmaf(wv.x, to_f(xr[0]), acc[r]);
        acc[r] = fmaf(wv.y, to_f(xr[1]), acc[r]);
        acc[r] = fmaf(wv.z, to_f(xr[2]), acc[r]);
        acc[r] = fmaf(wv.w, to_f(xr[3]), acc[r]);
      }
    }
#pragma unroll
    for (int r = 0; r < kRtTok; ++r) {
      const float v = warp_sum(acc[r]);
      if (lane == 0 && r < nt) out[(size_t)(t0 + r) * E + e] = v;
    }
  }
}

int moe_router_logits(const void* x, int x_is_f16, int ldx, const float* w, float* out, int T, int E, int H,
                      cudaStream_t st) {
  if (H % 4 || E < 1 || E > kMaxExperts || ldx < H) return -1;
  if (reinterpret_cast<uintptr_t>(w) & 15) return -3;
  if (T <= 0) return 0;
  const size_t smem = (size_t)kRtTok * H * 2;
  if (smem > 200 * 1024) return -2;
  dim3 grid((T + kRtTok - 1) / kRtTok, (E + kRtExp - 1) / kRtExp);
  cudaError_t e;
  if (x_is_f16) {
    auto k = moe_router_kernel<__half>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return -12;
    e = launch_pdl(k, grid, dim3(256), smem, st, static_cast<const __half*>(x), ldx, w, out, T, E, H);
  } else {
    auto k = moe_router_kernel<__nv_bfloat16>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess) return -12;
    e = launch_pdl(k, grid, dim3(256), smem, st, static_cast<const __nv_bfloat16*>(x), ldx, w, out, T, E, H);
  }
  return e == cudaSuccess ? 0 : -20;
}

__global__ void __launch_bounds__(256) moe_route_kernel(MoeRouteArgs a) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= a.T) return;
  const float* lg = a.logits + (size_t)t * a.E;
  constexpr int PER = kMaxExperts / 32;
  float p[PER];
  // gate probabilities (lane holds experts lane, lane+32, ...)
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int e = lane + 32 * i;
    p[i] = e < a.E ? lg[e] : -INFINITY;
    mx = fmaxf(mx, p[i]);
  }
  if (a.sigmoid) {
#pragma unroll
    for (int i = 0; i < PER; ++i) p[i] = (lane + 32 * i) < a.E ? 1.f / (1.f + __expf(-p[i])) : -INFINITY;
  } else {
    mx = warp_max(mx);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      p[i] = (lane + 32 * i) < a.E ? __expf(p[i] - mx) : 0.f;
      sum += p[i];
    }
    sum = warp_sum(sum);
    const float inv = 1.f / sum;
#pragma unroll
    for (int i = 0; i < PER; ++i) p[i] = (lane + 32 * i) < a.E ? p[i] * inv : -INFINITY;
  }
  // group-limited routing: experts outside the best topk_group groups (by their best expert) drop out
  if (a.n_group > 1 && a.topk_group < a.n_group) {
    const int gsz = a.E / a.n_group;
    __shared__ float gbest[8][64];
    for (int gi = 0; gi < a.n_group; ++gi) {
      float m = -INFINITY;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int e = lane + 32 * i;
        if (e < a.E && e / gsz == gi) m = fmaxf(m, p[i]);
      }
      m = warp_max(m);
      if (lane == 0) gbest[warp][gi] = m;
    }
    __syncwarp();
    unsigned long long keep = 0;  // groups kept (n_group <= 64)
    for (int r = 0; r < a.topk_group; ++r) {
      int best = -1;
      float bv = -INFINITY;
      for (int gi = 0; gi < a.n_group; ++gi)
        if (!((keep >> gi) & 1ull) && gbest[warp][gi] > bv) {
          bv = gbest[warp][gi];
          best = gi;
        }
      if (best >= 0) keep |= 1ull << best;
    }
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (e < a.E && !((keep >> (e / gsz)) & 1ull)) p[i] = -INFINITY;
    }
  }
  // top-k by repeated warp argmax (ties: lower expert id)
  int ids[kMaxTopK];
  float ws[kMaxTopK];
  float wsum = 0.f;
  for (int j = 0; j < a.k; ++j) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int e = lane + 32 * i;
      if (p[i] > bv || (p[i] == bv && e < be)) {
        bv = p[i];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    ids[j] = be;
    ws[j] = bv;
    wsum += bv;
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == be) p[i] = -INFINITY;
  }
  if (a.renorm) {
    const float inv = wsum > 0.f ? 1.f / wsum : 0.f;
    for (int j = 0; j < a.k; ++j) ws[j] *= inv;
  }
  if (a.ser_threshold > 0.f) {  // smart expert reduction: drop weak experts, renormalize the rest
    float s = 0.f;
    for (int j = 0; j < a.k; ++j) {
      if (j > 0 && ws[j] < a.ser_threshold) ws[j] = 0.f;
      s += ws[j];
    }
    const float inv = s > 0.f ? 1.f / s : 0.f;
    for (int j = 0; j < a.k; ++j) ws[j] *= inv;
  }
  if (lane == 0) {
    for (int j = 0; j < a.k; ++j) {
      const float wj = ws[j] * a.scale;
      a.ids[(size_t)t * a.k + j] = ids[j];
      a.weights[(size_t)t * a.k + j] = wj;
      if (ws[j] > 0.f) atomicAdd(a.counts + ids[j], 1);
    }
  }
}

__global__ void __launch_bounds__(256) moe_scan_kernel(MoeRouteArgs a) {
  pdl_wait();
  pdl_trigger();
  __shared__ int c[kMaxExperts];
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) c[e] = a.counts[e];
  __syncthreads();
  if (threadIdx.x == 0) {
    int run = 0;
    for (int e = 0; e < a.E; ++e) {
      a.off[e] = run;
      a.cursor[e] = run;
      run += c[e];
    }
    a.off[a.E] = run;
  }
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) a.counts[e] = 0;  // ready for the next call
}

template <typename T>
__global__ void __launch_bounds__(128) moe_dispatch_kernel(MoeRouteArgs a, const T* __restrict__ x,
                                                           T* __restrict__ xs) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x / a.k, j = blockIdx.x % a.k;
  const float wj = a.weights[(size_t)t * a.k + j];
  if (wj == 0.f) {  // dropped by SER
    if (threadIdx.x == 0) a.tok_row[(size_t)t * a.k + j] = -1;
    return;
  }
  __shared__ int row_s;
  if (threadIdx.x == 0) {
    const int e = a.ids[(size_t)t * a.k + j];
    const int row = atomicAdd(a.cursor + e, 1);
    a.row_tok[row] = t;
    a.row_w[row] = wj;
    a.tok_row[(size_t)t * a.k + j] = row;
    row_s = row;
  }
  __syncthreads();
  const int row = row_s;
  const int4* src = reinterpret_cast<const int4*>(x + (size_t)t * a.H);
  int4* dst = reinterpret_cast<int4*>(xs + (size_t)row * a.H);
  for (int i = threadIdx.x; i < a.H * (int)sizeof(T) / 16; i += blockDim.x) dst[i] = src[i];
}

// grid (T, ceil(H / 512)), 128 threads, 4 columns per thread
__global__ void __launch_bounds__(128) moe_combine_kernel(MoeCombineArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int n = (blockIdx.y * 128 + threadIdx.x) * 4;
  if (n >= a.H) return;
  const int lo = *a.lo, hi = *a.hi;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j = 0; j < a.k; ++j) {
    const int row = a.tok_row[(size_t)t * a.k + j];
    if (row < lo || row >= hi) continue;
    const float4 y = *reinterpret_cast<const float4*>(a.ys + (size_t)row * a.ld_ys + n);
    s.x += y.x;
    s.y += y.y;
    s.z += y.z;
    s.w += y.w;
  }
  float4* px = reinterpret_cast<float4*>(a.x + (size_t)t * a.ld_x + n);
  float4 v = *px;
  v.x += s.x;
  v.y += s.y;
  v.z += s.z;
  v.w += s.w;
  *px = v;
}

int moe_combine(const MoeCombineArgs& a, cudaStream_t st) {
  if (a.H % 4 || a.ld_ys % 4 || a.ld_x % 4 || (reinterpret_cast<uintptr_t>(a.ys) & 15) ||
      (reinterpret_cast<uintptr_t>(a.x) & 15))
    return -1;
  if (a.T <= 0) return 0;
  return launch_pdl(moe_combine_kernel, dim3(a.T, (a.H + 511) / 512), dim3(128), 0, st, a) == cudaSuccess ? 0 : -20;
}

int moe_route(const MoeRouteArgs& a, const void* x, int x_is_f16, void* xs, cudaStream_t st) {
  if (a.E <= 0 || a.E > kMaxExperts || a.k <= 0 || a.k > kMaxTopK || a.k > a.E) return -1;
  if (a.n_group > 64 || (a.n_group > 1 && a.E % a.n_group)) return -2;
  if ((a.H * 2) % 16) return -3;
  if (a.T <= 0) return 0;
  cudaError_t e = launch_pdl(moe_route_kernel, dim3((a.T + 7) / 8), dim3(256), 0, st, a);
  if (!xs) return e == cudaSuccess ? 0 : -20;  // routing only (expert parallel: ep_dispatch follows)
  if (e == cudaSuccess) e = launch_pdl(moe_scan_kernel, dim3(1), dim3(256), 0, st, a);
  if (e == cudaSuccess) {
    if (x_is_f16)
      e = launch_pdl(moe_dispatch_kernel<__half>, dim3(a.T * a.k), dim3(128), 0, st, a,
                     static_cast<const __half*>(x), static_cast<__half*>(xs));
    else
      e = launch_pdl(moe_dispatch_kernel<__nv_bfloat16>, dim3(a.T * a.k), dim3(128), 0, st, a,
                     static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(xs));
  }
  return e == cudaSuccess ? 0 : -20;
}

// ------------------------------------------------------------------ expert parallel (K5 / K7 across ranks)
// All-to-all over NVLink peer memory, no NCCL:
//   ep_counts_kernel    this rank's per-expert row counts -> every rank's count matrix, then a flag;
//   ep_dispatch_kernel  waits for every rank's counts, places each (token, slot) in the expert
//                       owner's receive rows (expert-major, then source rank) and copies the token
//                       row there with plain 16-byte stores; its last CTA flags every rank, waits
//                       for every rank's flag and writes this rank's receive offsets for the
//                       grouped expert GEMMs;
//   (grouped gate|up and down GEMMs on the received rows, outputs unweighted f32)
//   ep_signal_kernel    "my expert outputs are complete" to every rank;
//   ep_combine_kernel   each token row adds gate_weight * output of its slots, read from the expert
//                       owners over NVLink, in slot order (deterministic), into the residual stream.
// Buffer reuse needs no barrier: a peer writes this rank's receive rows or count row for the next
// layer only after its combine of this layer, which waited for this rank's outputs, which this
// rank computed after reading its receive rows.
namespace {

BARQ_DEV uint32_t ep_cur(const EpArgs& a) { return *a.epoch + 1; }

// receive row of the first row that source `src` sends to expert e (on e's owner)
BARQ_DEV int ep_base(const int* cm, int W, int E, int E_local, int e, int src) {
  const int e0 = (e / E_local) * E_local;
  int b = 0;
  for (int x = e0; x < e; ++x)
    for (int r = 0; r < W; ++r) b += cm[r * E + x];
  for (int r = 0; r < src; ++r) b += cm[r * E + e];
  return b;
}

}  // namespace

__global__ void __launch_bounds__(256) ep_counts_kernel(EpArgs a) {
  const uint32_t ep = ep_cur(a);
  for (int i = threadIdx.x; i < a.W * a.E; i += blockDim.x) {
    const int q = i / a.E, e = i - q * a.E;
    a.cnt_all[q][a.rank * a.E + e] = a.counts[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < a.W) st_release_sys(a.cnt_flags[threadIdx.x] + a.rank, ep);
}

// grid: one CTA per own token row (at least 1), 128 threads
template <typename T>
__global__ void __launch_bounds__(128) ep_dispatch_kernel(EpArgs a) {
  const uint32_t ep = ep_cur(a);
  __shared__ int cm[kSpMaxRanks * kMaxExperts];
  __shared__ int pos_s[kMaxTopK], dst_s[kMaxTopK];
  __shared__ int last_s;
  // every rank's counts (the local row was written by ep_counts_kernel before this launch)
  if (threadIdx.x < a.W && !wait_epoch_sys(a.cnt_flags[a.rank] + threadIdx.x, ep, a.wait_ns))
    atomicExch(a.err, 0x700 | threadIdx.x);
  __syncthreads();
  const int* own = a.cnt_all[a.rank];
  for (int i = threadIdx.x; i < a.W * a.E; i += blockDim.x) cm[i] = __ldcg(own + i);
  __syncthreads();
  const int t = blockIdx.x;
  if (t < a.rows) {
    if (threadIdx.x < a.k) {
      const int j = threadIdx.x;
      const int e = a.ids[(size_t)t * a.k + j];
      int dst = -1, pos = 0;
      if (a.weights[(size_t)t * a.k + j] > 0.f) {
        dst = e / a.E_local;
        pos = ep_base(cm, a.W, a.E, a.E_local, e, a.rank) + atomicAdd(a.cursor + e, 1);
      }
      pos_s[j] = pos;
      dst_s[j] = dst;
      a.disp_pos[(size_t)t * a.k + j] = make_int2(dst, pos);
    }
    __syncthreads();
    const int4* src = reinterpret_cast<const int4*>(static_cast<const T*>(a.x) + (size_t)t * a.H);
    const int n16 = a.H * (int)sizeof(T) / 16;
    for (int j = 0; j < a.k; ++j) {
      if (dst_s[j] < 0) continue;
      int4* d = reinterpret_cast<int4*>(static_cast<T*>(a.recv_x[dst_s[j]]) + (size_t)pos_s[j] * a.H);
      for (int i = threadIdx.x; i < n16; i += blockDim.x) d[i] = src[i];  // NVLink stores
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) last_s = atom_add_acq_rel_gpu(a.done, 1) == (int)gridDim.x - 1;
  __syncthreads();
  if (!last_s) return;
  // last CTA: every row of this rank is out; flag every rank, then wait for every rank's rows
  if (threadIdx.x < a.E) {
    a.cursor[threadIdx.x] = 0;
    a.counts[threadIdx.x] = 0;
  }
  for (int e = threadIdx.x + 128; e < a.E; e += 128) {
    a.cursor[e] = 0;
    a.counts[e] = 0;
  }
  if (threadIdx.x < a.W) st_release_sys(a.disp_flags[threadIdx.x] + a.rank, ep);
  if (threadIdx.x <= a.E_local) {
    const int e = a.rank * a.E_local + threadIdx.x;
    a.recv_off[threadIdx.x] = threadIdx.x == a.E_local
                                  ? ep_base(cm, a.W, a.E, a.E_local, e - 1, a.W)
                                  : ep_base(cm, a.W, a.E, a.E_local, e, 0);
  }
  if (threadIdx.x < a.W && !wait_epoch_sys(a.disp_flags[a.rank] + threadIdx.x, ep, a.wait_ns))
    atomicExch(a.err, 0x800 | threadIdx.x);
  if (threadIdx.x == 0) *a.done = 0;
}

__global__ void __launch_bounds__(32) ep_signal_kernel(EpArgs a) {
  const uint32_t ep = ep_cur(a);
  __threadfence_system();  // this rank's expert outputs (previous kernel) before the flags
  if (threadIdx.x < a.W) st_release_sys(a.ys_flags[threadIdx.x] + a.rank, ep);
}

// grid: (one CTA per own token row (at least 1), ceil(H / 512)), 128 threads, 4 columns each
__global__ void __launch_bounds__(128) ep_combine_kernel(EpArgs a) {
  const uint32_t ep = ep_cur(a);
  __shared__ int last_s;
  if (threadIdx.x < a.W && !wait_epoch_sys(a.ys_flags[a.rank] + threadIdx.x, ep, a.wait_ns))
    atomicExch(a.err, 0x900 | threadIdx.x);
  __syncthreads();
  const int t = blockIdx.x, n = (blockIdx.y * 128 + threadIdx.x) * 4;
  if (t < a.rows && n < a.H) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < a.k; ++j) {  // slot order: the same bits whatever order rows arrived in
      const int2 dp = a.disp_pos[(size_t)t * a.k + j];
      if (dp.x < 0) continue;
      const float w = a.weights[(size_t)t * a.k + j];
      const float4 y = __ldcg(reinterpret_cast<const float4*>(a.ys[dp.x] + (size_t)dp.y * a.H + n));
      s.x += w * y.x;
      s.y += w * y.y;
      s.z += w * y.z;
      s.w += w * y.w;
    }
    float4* px = reinterpret_cast<float4*>(a.out + (size_t)t * a.H + n);
    float4 v = *px;
    v.x += s.x;
    v.y += s.y;
    v.z += s.z;
    v.w += s.w;
    *px = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) last_s = atom_add_acq_rel_gpu(a.done + 1, 1) == (int)(gridDim.x * gridDim.y) - 1;
  __syncthreads();
  if (last_s && threadIdx.x == 0) {
    a.done[1] = 0;
    *a.epoch = ep;
  }
}

static bool ep_ok(const EpArgs& a) {
  if (a.W < 1 || a.W > kSpMaxRanks || a.rank < 0 || a.rank >= a.W || a.E <= 0 || a.E > kMaxExperts ||
      a.E_local * a.W != a.E || a.E_local > 127 || a.k <= 0 || a.k > kMaxTopK || a.H % 8 || a.rows < 0)
    return false;
  for (int q = 0; q < a.W; ++q)
    if (!a.cnt_all[q] || !a.cnt_flags[q] || !a.recv_x[q] || !a.disp_flags[q] || !a.ys[q] || !a.ys_flags[q] ||
        (reinterpret_cast<uintptr_t>(a.recv_x[q]) & 15) || (reinterpret_cast<uintptr_t>(a.ys[q]) & 15))
      return false;
  return true;
}

int ep_dispatch(const EpArgs& a, int x_is_f16, cudaStream_t st) {
  if (!ep_ok(a) || (reinterpret_cast<uintptr_t>(a.x) & 15)) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = st;
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(256);
  if (cudaLaunchKernelEx(&cfg, ep_counts_kernel, a) != cudaSuccess) return -20;
  cfg.gridDim = dim3(a.rows > 0 ? a.rows : 1);
  cfg.blockDim = dim3(128);
  const cudaError_t e = x_is_f16 ? cudaLaunchKernelEx(&cfg, ep_dispatch_kernel<__half>, a)
                                 : cudaLaunchKernelEx(&cfg, ep_dispatch_kernel<__nv_bfloat16>, a);
  return e == cudaSuccess ? 0 : -20;
}

int ep_combine(const EpArgs& a, cudaStream_t st) {
  if (!ep_ok(a) || (reinterpret_cast<uintptr_t>(a.out) & 15)) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = st;
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(32);
  if (cudaLaunchKernelEx(&cfg, ep_signal_kernel, a) != cudaSuccess) return -20;
  cfg.gridDim = dim3(a.rows > 0 ? a.rows : 1, (a.H + 511) / 512);
  cfg.blockDim = dim3(128);
  return cudaLaunchKernelEx(&cfg, ep_combine_kernel, a) == cudaSuccess ? 0 : -20;
}

}  // namespace barq
