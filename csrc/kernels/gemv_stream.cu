// K1b: streaming quantized GEMV for decode (1..8 tokens): persistent, bulk-copy fed, stream-K.
//
// The reference's decode matmul is a host round trip (backend/src/cuda_quant.rs:104-126); this is
// the B200 path for the same y = W x with W in GGUF blocks and x as int8 (ActQ8).
//
// Why a second GEMV: with K = 4096 a warp-per-row GEMV gives each lane only a few dependent DRAM
// round trips, so it is latency-bound (~1.5 TB/s).  Here one CTA per SM walks a contiguous range of
// weight chunks (the tiled layout makes "128 rows x G columns" one contiguous chunk, and a range of
// chunks one contiguous span of memory):
//   warp 8 (one thread)  cp.async.bulk of whole chunks into an S-deep shared-memory ring
//                        (~180 KB in flight per SM, enough to cover DRAM latency at full rate);
//   warps 0-7            dp4a against the int8 activations: warp w takes rows 32*(w/2) + lane and
//                        half w%2 of each chunk row (warp-uniform, so no divergence); the two
//                        halves of a row meet in shared memory once per row tile.
// Work units are (row tile, K chunk) pairs split evenly over the CTAs ("stream-K"), so every SM
// streams the same number of bytes.  A row tile finished by one CTA is written directly; a tile
// shared by several CTAs is combined in an f32 workspace: each stores its partial sums in a slot of
// its own, the last to arrive (per-tile counter) adds the slots in a fixed order, applies the
// epilogue and clears the counter again (the next call or CUDA-graph replay finds it zero).  No
// floating-point atomics: a decode step gives the same bits on every run.
// Epilogues: STORE_F32, ADD_F32, STORE_BF16,
// SWIGLU_Q8 (rows interleaved [32 gate | 32 up]; writes silu(g)*u as int8 activations), and
// AR_PUSH: the tensor-parallel all-reduce of a row-parallel layer fused into the GEMV.  The CTA
// that finishes a 128-row tile stores it at once into every peer's receive buffer (slot = this
// rank) over NVLink, each value packed with the call's epoch into one 64-bit store, so no memory
// fence or flag is needed: a reader that sees the epoch sees the value (the low-latency protocol
// of NCCL's LL mode).  It then waits for the same tile of every peer in its own receive buffer
// (bounded by %globaltimer) and adds the world's sum into the residual stream.  Every rank splits
// the work identically, so tile t's exchange only waits on the peers' tile t; no separate
// all-reduce launch and no NCCL call on the decode path.
// Every mbarrier wait is bounded; on expiry the CTA records an error word and unwinds.
#include <cstdlib>

#include "gemv_traits.cuh"
#include "launch.h"
#include "pdl.cuh"
#include "sysflags.cuh"
#include "tc_common.cuh"

namespace barq {

using namespace tc;

namespace {

constexpr int kRingBytes = 184 * 1024;
constexpr int kNormMaxK = 4096;
constexpr int kSlotFloats = 8 * 128;  // one partial row tile (up to 8 tokens) per workspace slot  // fused-RMSNorm prologue: longest activation row staged in smem

// Compute warps per CTA: 16 (each row split over 4 warps) for 1-2 tokens, where latency hiding
// matters most and registers allow it; 8 (rows split over 2 warps) otherwise and for formats
// with 64-column chunks (two 32-weight parts per chunk row).
template <int WT, int BS>
struct StreamCfg {
  static constexpr int NP = TileFmt<WT>::G / 32;
  static constexpr int TPR = (BS <= 2 && NP >= 8) ? 4 : 2;  // warps per row group
  static constexpr int NW = 4 * TPR;                        // compute warps: 4 row groups of 32
  static constexpr int THREADS = (NW + 1) * 32;
  // 1-2 tokens: room for the fused-norm activations (q, ql, s, dl per token) after the ring
  static constexpr int XS_BYTES = BS <= 2 ? BS * (2 * kNormMaxK + 2 * (kNormMaxK / 32) * 8) : 0;
  static constexpr int RING = kRingBytes - XS_BYTES;
  static constexpr int S = RING / TileFmt<WT>::CHUNK > 32 ? 32 : RING / TileFmt<WT>::CHUNK;
};

BARQ_DEV void bulk_copy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

template <int NW>
BARQ_DEV void compute_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NW * 32) : "memory");
}

// Optional prologue: the activation is rmsnorm(h) * w quantized to int8 inside the kernel (each CTA
// recomputes it into shared memory while its weight stream is already in flight), replacing a
// separate RMSNorm launch.  h: f32 [B, K]; null = activations come in x.
struct NormIn {
  const float* h;
  const float* w;
  float eps;
  int x2;
};

struct StreamWs {
  float* acc;  // [grid + tiles][8 * 128] f32 partial sums of shared row tiles (slot per CTA piece)
  int* cnt;    // [N / 128] units accumulated per row tile (zero between calls)
  int* err;
  int exp;  // diagnostics: bit 0 = compute warps skip the arithmetic (still wait for and release chunks);
            // AR_PUSH: bit 1 = skip the flag exchange, bit 2 = skip the final reduction
};

}  // namespace

template <class T, int WT, int BS, bool X2>
__global__ void __launch_bounds__(StreamCfg<WT, BS>::THREADS, 1)
    qgemv_stream_kernel(QW w, ActQ8 x, int B, GemvEpi ep, StreamWs ws, NormIn ni, ArPush ar) {
  using F = TileFmt<WT>;
  using Cfg = StreamCfg<WT, BS>;
  constexpr int CH = F::CHUNK;
  constexpr int S = Cfg::S;
  constexpr int NP = Cfg::NP;     // 32-weight parts per chunk row
  constexpr int TPR = Cfg::TPR;   // warps sharing a row group
  constexpr int NW = Cfg::NW;
  constexpr int PPT = NP / TPR;   // parts per thread
  static_assert(NP % TPR == 0, "whole parts per thread");
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t full[S], empty[S];
  __shared__ float red[128][BS];
  __shared__ float comb[TPR - 1][128][BS];
  __shared__ int last_s;
  __shared__ float red_ss[NW];
  __shared__ int err_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KG = w.K / F::G;
  const int tiles = (w.N + 127) / 128;
  const int U = tiles * KG;  // < 2^31 for any weight this library loads
  const int u0 = (int)((long long)U * blockIdx.x / gridDim.x), u1 = (int)((long long)U * (blockIdx.x + 1) / gridDim.x);
  const int n_units = u1 - u0;
  const int nparts = w.K >> 5;
  if (threadIdx.x == 0) {
    err_s = 0;
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], NW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  volatile int* err = &err_s;
  // Weights do not depend on earlier kernels: the producer streams them at once.  The compute warps
  // wait for the previous kernel (activations, output buffers, workspace) before their first read.
  pdl_trigger();

  if (warp == NW) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      const uint8_t* src = w.p0 + (size_t)u0 * CH;
      int issued = 0, s = 0;
      uint32_t ph = 0;
      for (int i = 0; i < n_units; ++i) {
        if (i >= S && !mbar_wait(&empty[s], ph ^ 1, err, 1)) break;
        mbar_expect_tx(&full[s], CH);
        bulk_copy(smem + s * CH, src, CH, &full[s]);
        src += CH;
        issued = i + 1;
        if (++s == S) {
          s = 0;
          ph ^= 1;
        }
      }
      // Before the CTA may exit, every copy issued must have landed (normally the compute warps
      // already saw each one; after an error this waits, bounded, for the ones in flight).
      for (int i = issued > S ? issued - S : 0; i < issued; ++i)
        mbar_wait_bounded(&full[i % S], (uint32_t)((i / S) & 1));
    }
  } else {
    // ------------------------------------------------------------------ compute
    pdl_wait();
    if (Cfg::XS_BYTES > 0 && ni.h) {
      // fused RMSNorm + int8 quantization of the B activation rows into shared memory
      const int K = w.K, G32 = w.K / 32;
      int8_t* sq = reinterpret_cast<int8_t*>(smem + S * CH);
      int8_t* sql = sq + BS * K;
      float2* ssc = reinterpret_cast<float2*>(sql + BS * K);
      float2* sdl = ssc + BS * G32;
      for (int b = 0; b < B; ++b) {
        const float* hb = ni.h + (size_t)b * K;
        float ss = 0.f;
        for (int k = threadIdx.x; k < K; k += NW * 32) {
          const float v = hb[k];
          ss += v * v;
        }
        ss = warp_sum(ss);
        if (lane == 0) red_ss[warp] = ss;
        compute_sync<NW>();
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < NW; ++i) tot += red_ss[i];
        const float rstd = rsqrtf(tot / (float)K + ni.eps);
        const ActOut o{sq + b * K, ssc + b * G32, ni.x2 ? sql + b * K : nullptr, ni.x2 ? sdl + b * G32 : nullptr};
        for (int g = warp; g < G32; g += NW) {
          const int k = g * 32 + lane;
          act_store32(o, hb[k] * rstd * ni.w[k], k, g, lane);
        }
        compute_sync<NW>();  // red_ss reused by the next row
      }
      x = ActQ8{sq, ssc, ni.x2 ? sql : nullptr, ni.x2 ? sdl : nullptr};
    }
    uint32_t ar_ep = 0;  // AR_PUSH: this call's epoch (the counter is advanced by the last CTA out)
    if (ep.mode == EPI_AR_PUSH) ar_ep = *ar.epoch + 1;
    const int half = warp % TPR, r = (warp / TPR) * 32 + lane;  // half: this warp's slice of the row
    const int tid = threadIdx.x;
    float acc[BS];
#pragma unroll
    for (int b = 0; b < BS; ++b) acc[b] = 0.f;
    int tile_first = u0;  // first unit of the current tile inside this CTA's range
    int tile = u0 / KG, kg = u0 - (u0 / KG) * KG, s = 0;
    uint32_t ph = 0;
    for (int i = 0; i < n_units; ++i, ++kg) {
      if (kg == KG) {
        kg = 0;
        ++tile;
      }
      if (i > 0 && ++s == S) {
        s = 0;
        ph ^= 1;
      }
      const int u = u0 + i;
      // On an error the loop keeps running (without waiting) so that every compute warp still
      // reaches each named barrier below; the results are discarded by the host.
      const bool have = !*err && mbar_wait(&full[s], ph, err, 2);
      const uint8_t* ch = smem + s * CH;
      const int row = tile * 128 + r;
      if (have && !(kDiag && (ws.exp & 1))) {
        if constexpr (WT == W_Q4_K || WT == W_Q5_K || WT == W_Q6_K) {
          switch (half) {
            case 0: T::template chunk_dot<0 * PPT, PPT, BS, X2>(ch, r, kg, x, w.K, nparts, B, acc); break;
            case 1: T::template chunk_dot<1 * PPT, PPT, BS, X2>(ch, r, kg, x, w.K, nparts, B, acc); break;
            case 2: T::template chunk_dot<(TPR > 2 ? 2 : 0) * PPT, PPT, BS, X2>(ch, r, kg, x, w.K, nparts, B, acc); break;
            default: T::template chunk_dot<(TPR > 2 ? 3 : 0) * PPT, PPT, BS, X2>(ch, r, kg, x, w.K, nparts, B, acc); break;
          }
        } else {
#pragma unroll
          for (int j = 0; j < PPT; ++j) {
            const int q = half * PPT + j;
            const typename T::W wq = T::load_s(ch, r, q);
            const int p = kg * NP + q;
#pragma unroll
            for (int b = 0; b < BS; ++b) {
              if (b < B) {
                acc[b] += T::dot(wq, T::load_x(x.q + (size_t)b * w.K, x.s + (size_t)b * nparts, p), q);
                if (X2) acc[b] += T::dot(wq, T::load_x(x.ql + (size_t)b * w.K, x.dl + (size_t)b * nparts, p), q);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (kg != KG - 1 && i != n_units - 1) continue;

      // ---- tile done (or this CTA's range ends inside it)
      if (half) {
#pragma unroll
        for (int b = 0; b < BS; ++b) comb[half - 1][r][b] = acc[b];
      }
      compute_sync<NW>();
      if (!half) {
#pragma unroll
        for (int t = 0; t < TPR - 1; ++t)
#pragma unroll
          for (int b = 0; b < BS; ++b) acc[b] += comb[t][r][b];
      }
      const int tu0 = tile * KG;
      const bool whole = tile_first == tu0 && u == tu0 + KG - 1;
      const int covered = (int)(u - tile_first + 1);
      tile_first = u + 1;
      const bool valid = row < w.N;
      bool emit = whole;
      if (!whole) {
        // Shared tile: every contributing CTA stores its partial sums in its own workspace slot
        // (slot = CTA + tile, unique because both grow along the unit sequence); the last CTA to
        // arrive sums the slots in CTA order, so the result does not depend on arrival order.
        if (half == 0 && valid)
#pragma unroll
          for (int b = 0; b < BS; ++b)
            if (b < B) ws.acc[(size_t)(blockIdx.x + tile) * kSlotFloats + b * 128 + r] = acc[b];
        __threadfence();
        compute_sync<NW>();
        if (tid == 0) last_s = atomicAdd(ws.cnt + tile, covered) + covered == KG;
        compute_sync<NW>();
        emit = last_s != 0;
        if (emit) {
          __threadfence();
          const long long G = gridDim.x;
          const int c_first = (int)(((long long)(tu0 + 1) * G + U - 1) / U) - 1;
          const int c_last = (int)(((long long)(tu0 + KG) * G + U - 1) / U) - 1;
          if (half == 0 && valid) {
            // pieces in CTA order; the BS loads of one piece are issued together
#pragma unroll
            for (int b = 0; b < BS; ++b) acc[b] = 0.f;
            for (int c = c_first; c <= c_last; ++c) {
              const float* slot = ws.acc + (size_t)(c + tile) * kSlotFloats + r;
              float v[BS];
#pragma unroll
              for (int b = 0; b < BS; ++b) v[b] = b < B ? __ldcg(slot + b * 128) : 0.f;
#pragma unroll
              for (int b = 0; b < BS; ++b) acc[b] += v[b];
            }
          }
          if (tid == 0) ws.cnt[tile] = 0;
        }
      }
      if (emit) {
        if (ep.mode == EPI_SWIGLU_Q8) {
          if (half == 0)
#pragma unroll
            for (int b = 0; b < BS; ++b) red[r][b] = acc[b];
          compute_sync<NW>();
          if (warp < 2) {  // group `warp`: gate rows 64*warp + [0,32), up rows 64*warp + 32 + [0,32)
            const int n_out = w.N / 2;
            const int o = tile * 64 + warp * 32 + lane;
            for (int b = 0; b < B; ++b) {
              const float g = red[warp * 64 + lane][b], up = red[warp * 64 + 32 + lane][b];
              const float h = silu(g) * up;
              act_store32(ep.out_q, h, (size_t)b * n_out + o, (size_t)b * (n_out / 32) + tile * 2 + warp, lane);
              if (ep.out_bf16) ep.out_bf16[(size_t)b * ep.ld_out + o] = __float2bfloat16(h);
            }
          }
          compute_sync<NW>();
        } else if (half == 0 && valid) {
#pragma unroll
          for (int b = 0; b < BS; ++b) {
            if (b >= B) break;
            float v = acc[b] + (ep.bias ? ep.bias[row] : 0.f);
            const size_t idx = (size_t)b * ep.ld_out + row;
            if (ep.mode == EPI_AR_PUSH) {
              // (epoch, value) in one 64-bit store: a peer that sees the epoch sees the value
              const size_t o = ((size_t)ar.rank * B + b) * w.N + row;
              const uint64_t pk = ((uint64_t)ar_ep << 32) | __float_as_uint(v);
              if (!ar.skip_signal)
                for (int q = 0; q < ar.world; ++q)
                  if (q != ar.rank) st_relaxed_sys_u64(ar.dst[q] + o, pk);  // NVLink store
              red[r][b] = v;
            } else if (ep.mode == EPI_ADD_F32)
              ep.out_f32[idx] += v;
            else if (ep.mode == EPI_STORE_F32)
              ep.out_f32[idx] = v;
            else
              ep.out_bf16[idx] = __float2bfloat16(v);
          }
          if (ep.mode == EPI_AR_PUSH) {
            // the same tile of every peer: wait for its (epoch, value) words in this GPU's
            // receive buffer, then add the world's sum into the residual stream
            const uint64_t* own = ar.dst[ar.rank];
            for (int b = 0; b < B; ++b) {
              // summed in rank order on every rank, so the replicated residual stays bit-identical
              // across ranks for any world size (own-value-first order differs per rank from 3 on)
              float sum = 0.f;
              bool ok = true;
              for (int q = 0; q < ar.world && ok; ++q) {
                if (q == ar.rank) {
                  sum += red[r][b];
                  continue;
                }
                uint64_t pk = 0;
                ok = wait_pair_sys(own + ((size_t)q * B + b) * w.N + row, ar_ep, ar.wait_ns, ws.err,
                                   pk);
                if (ok)
                  sum += __uint_as_float((uint32_t)pk);
                else
                  atomicExch(ws.err, 0x300 | q);
              }
              if (ok) ar.x[(size_t)b * ar.ld_x + row] += sum;
            }
          }
        }
      }
      compute_sync<NW>();  // comb[] / red[] are free again for the next row tile
#pragma unroll
      for (int b = 0; b < BS; ++b) acc[b] = 0.f;
    }
    if (ep.mode == EPI_AR_PUSH) {
      // every CTA has read the epoch (program order before its acq_rel count): the last one out
      // advances it and clears the counter for the next call / graph replay
      compute_sync<NW>();
      if (tid == 0 && atom_add_acq_rel_gpu(ar.done, 1) == (int)gridDim.x - 1) {
        *ar.done = 0;
        *ar.epoch = ar_ep;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && err_s && ws.err) atomicExch(ws.err, err_s);
}

namespace {

template <class T, int WT, int BS, bool X2>
int launch_stream(const QW& w, const ActQ8& x, int B, const GemvEpi& ep, const StreamWs& ws, const NormIn& ni,
                  const ArPush& ar, int n_sm, cudaStream_t st) {
  using F = TileFmt<WT>;
  using Cfg = StreamCfg<WT, BS>;
  if (ni.h && (Cfg::XS_BYTES == 0 || w.K > kNormMaxK)) return -6;
  const int smem = Cfg::S * F::CHUNK + Cfg::XS_BYTES;
  auto kern = qgemv_stream_kernel<T, WT, BS, X2>;
  constexpr int THREADS = StreamCfg<WT, BS>::THREADS;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const long U = (long)((w.N + 127) / 128) * (w.K / F::G);
  int grid = (int)(U < n_sm ? U : n_sm);
  if (grid > 256) grid = 256;  // workspace slots: CTA + tile < 256 + tiles (qgemv_stream_ws_floats)
  return launch_pdl(kern, dim3(grid), dim3(THREADS), (size_t)smem, st, w, x, B, ep, ws, ni, ar) == cudaSuccess ? 0 : -20;
}

template <class T, int WT, int BS>
int launch_stream_x(const QW& w, const ActQ8& x, int B, const GemvEpi& ep, const StreamWs& ws, const NormIn& ni,
                    const ArPush& ar, int n_sm, cudaStream_t st) {
  const bool x2 = ni.h ? ni.x2 != 0 : x.ql != nullptr;
  return x2 ? launch_stream<T, WT, BS, true>(w, x, B, ep, ws, ni, ar, n_sm, st)
            : launch_stream<T, WT, BS, false>(w, x, B, ep, ws, ni, ar, n_sm, st);
}

template <class T, int WT>
int launch_stream_b(const QW& w, const ActQ8& x, int B, const GemvEpi& ep, const StreamWs& ws, const NormIn& ni,
                    const ArPush& ar, int n_sm, cudaStream_t st) {
  if (B <= 1) return launch_stream_x<T, WT, 1>(w, x, B, ep, ws, ni, ar, n_sm, st);
  if (B <= 2) return launch_stream_x<T, WT, 2>(w, x, B, ep, ws, ni, ar, n_sm, st);
  if (B <= 4) return launch_stream_x<T, WT, 4>(w, x, B, ep, ws, ni, ar, n_sm, st);
  return launch_stream_x<T, WT, 8>(w, x, B, ep, ws, ni, ar, n_sm, st);
}

}  // namespace

int qgemv_stream(const QW& w, const ActQ8& x, int B, const GemvEpi& ep, float* ws_acc, int* ws_cnt, int* err,
                 const float* norm_h, const float* norm_w, float norm_eps, int norm_x2, cudaStream_t st,
                 const ArPush* ar) {
  const NormIn ni{norm_h, norm_w, norm_eps, norm_x2};
  ArPush arp{};
  if (ep.mode == EPI_AR_PUSH) {
    if (!ar || ar->world < 1 || ar->world > kArMaxRanks || ar->rank < 0 || ar->rank >= ar->world || !ar->x ||
        !ar->epoch || !ar->done || (w.N % 128) || (ar->ld_x % 4) || (reinterpret_cast<uintptr_t>(ar->x) & 15))
      return -7;
    if (!ar->dst) return -7;
    arp = *ar;
  }
  if (B < 1 || B > 8) return -1;
  if (ep.mode == EPI_SWIGLU_Q8 && (w.N % 128)) return -3;
  if ((reinterpret_cast<uintptr_t>(w.p0) & 15)) return -4;
  static int n_sm = 0;
  if (!n_sm) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    if (n_sm <= 0) n_sm = 148;
  }
  static const int exp_flags = [] {
    const char* e = getenv("BARQ_GEMV_EXP");
    return e ? atoi(e) : 0;
  }();
  const StreamWs ws{ws_acc, ws_cnt, err, exp_flags};
  switch (w.type) {
    case W_Q4_0: if (w.K % 64) return -2; return launch_stream_b<T4Block<false>, W_Q4_0>(w, x, B, ep, ws, ni, arp, n_sm, st);
    case W_IQ4_NL: if (w.K % 64) return -2; return launch_stream_b<T4Block<true>, W_IQ4_NL>(w, x, B, ep, ws, ni, arp, n_sm, st);
    case W_Q8_0: if (w.K % 64) return -2; return launch_stream_b<TQ8_0, W_Q8_0>(w, x, B, ep, ws, ni, arp, n_sm, st);
    case W_Q4_K: if (w.K % 256) return -2; return launch_stream_b<TK45<false>, W_Q4_K>(w, x, B, ep, ws, ni, arp, n_sm, st);
    case W_Q5_K: if (w.K % 256) return -2; return launch_stream_b<TK45<true>, W_Q5_K>(w, x, B, ep, ws, ni, arp, n_sm, st);
    case W_Q6_K: if (w.K % 256) return -2; return launch_stream_b<TQ6_K, W_Q6_K>(w, x, B, ep, ws, ni, arp, n_sm, st);
  }
  return -5;
}

}  // namespace barq
