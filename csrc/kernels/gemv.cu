// K1: quantized GEMV for decode (1..8 tokens), dp4a on int8 activations.
//
// Replaces the reference's host-fallback "CUDA" quantized matmul
// (backend/src/cuda_quant.rs:104-126, 240-338), which copies to the host and multiplies there.
//
// Layout: a warp owns RW consecutive weight rows; its lanes split K into 32-weight parts (see
// gemv_traits.cuh), so each weight byte is read exactly once, coalesced, with an evict-first hint.
// The activation parts a lane needs are loaded once and reused across the RW rows.  Partial sums
// are reduced with warp shuffles; the epilogue is chosen at run time:
//   EPI_STORE_F32  out[b, n] = acc (+ bias)
//   EPI_ADD_F32    out[b, n] += acc             (residual stream update, o_proj / down_proj)
//   EPI_STORE_BF16 out[b, n] = bf16(acc (+ bias))
//   EPI_SWIGLU_Q8  CTA holds 32 gate rows + 32 matching up rows; writes silu(g)*u for 32 outputs
//                  straight into the int8 activation layout of the next GEMV (and optionally bf16).
#include "gemv_traits.cuh"
#include "pdl.cuh"
#include "launch.h"

namespace barq {

template <class T, int BS, int RW, int NW, bool X2>
__global__ void __launch_bounds__(NW * 32) qgemv_kernel(QW w, ActQ8 x, int B, GemvEpi ep) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * NW + warp) * RW;
  const int K = w.K;
  const int nparts = K >> 5;
  float acc[RW][BS];
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int b = 0; b < BS; ++b) acc[r][b] = 0.f;

  const int8_t* xq = x.q;
  const float2* xs = x.s;
#pragma unroll 2
  for (int p = lane; p < nparts; p += 32) {
    typename T::W wr[RW];
#pragma unroll
    for (int r = 0; r < RW; ++r) {
      int row = min(row0 + r, w.N - 1);
      wr[r] = T::load_w(w, row, p);
    }
#pragma unroll
    for (int b = 0; b < BS; ++b) {
      if (b < B) {
        typename T::X xr = T::load_x(xq + (size_t)b * K, xs + (size_t)b * nparts, p);
#pragma unroll
        for (int r = 0; r < RW; ++r) acc[r][b] += T::dot(wr[r], xr, lane);
        if (X2) {  // second (residual) activation term
          typename T::X xl = T::load_x(x.ql + (size_t)b * K, x.dl + (size_t)b * nparts, p);
#pragma unroll
          for (int r = 0; r < RW; ++r) acc[r][b] += T::dot(wr[r], xl, lane);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < RW; ++r)
#pragma unroll
    for (int b = 0; b < BS; ++b) acc[r][b] = warp_sum(acc[r][b]);

  if (ep.mode == EPI_SWIGLU_Q8) {
    // rows of this CTA: [32 gate | 32 up] for outputs 32*blockIdx.x + [0, 32)
    __shared__ float red[NW * RW][BS];
    if (lane == 0) {
#pragma unroll
      for (int r = 0; r < RW; ++r)
#pragma unroll
        for (int b = 0; b < BS; ++b) red[warp * RW + r][b] = acc[r][b];
    }
    __syncthreads();
    if (warp == 0) {
      const int n_out = w.N / 2;
      const int o = blockIdx.x * 32 + lane;
      for (int b = 0; b < B; ++b) {
        float g = red[lane][b], u = red[32 + lane][b];
        float h = silu(g) * u;
        act_store32(ep.out_q, h, (size_t)b * n_out + o, (size_t)b * (n_out / 32) + blockIdx.x, lane);
        if (ep.out_bf16) ep.out_bf16[(size_t)b * ep.ld_out + o] = __float2bfloat16(h);
      }
    }
    return;
  }
  // Lane (r * BS + b) writes value (r, b).
#pragma unroll
  for (int r = 0; r < RW; ++r) {
#pragma unroll
    for (int b = 0; b < BS; ++b) {
      const int row = row0 + r;
      if (lane == ((r * BS + b) & 31) && b < B && row < w.N) {
        float v = acc[r][b];
        if (ep.bias) v += ep.bias[row];
        size_t idx = (size_t)b * ep.ld_out + row;
        if (ep.mode == EPI_ADD_F32)
          ep.out_f32[idx] += v;
        else if (ep.mode == EPI_STORE_F32)
          ep.out_f32[idx] = v;
        else
          ep.out_bf16[idx] = __float2bfloat16(v);
      }
    }
  }
}

// Dense bf16 weight GEMV (fallback for rows whose length is not a multiple of 32, e.g. F16/F32
// GGUF tensors converted at load).  x is bf16 [B, K].
template <int BS>
__global__ void __launch_bounds__(128) bf16_gemv_kernel(const __nv_bfloat16* __restrict__ W, int N, int K,
                                                        const __nv_bfloat16* __restrict__ x, int ldx, int B,
                                                        GemvEpi ep) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  if (row >= N) return;
  float acc[BS];
#pragma unroll
  for (int b = 0; b < BS; ++b) acc[b] = 0.f;
  const __nv_bfloat16* wr = W + (size_t)row * K;
  for (int k = lane; k < K; k += 32) {
    float wv = __bfloat162float(wr[k]);
#pragma unroll
    for (int b = 0; b < BS; ++b)
      if (b < B) acc[b] += wv * __bfloat162float(x[(size_t)b * ldx + k]);
  }
#pragma unroll
  for (int b = 0; b < BS; ++b) acc[b] = warp_sum(acc[b]);
  if (lane == 0) {
    for (int b = 0; b < B; ++b) {
      float v = acc[b] + (ep.bias ? ep.bias[row] : 0.f);
      size_t idx = (size_t)b * ep.ld_out + row;
      if (ep.mode == EPI_ADD_F32)
        ep.out_f32[idx] += v;
      else if (ep.mode == EPI_STORE_F32)
        ep.out_f32[idx] = v;
      else
        ep.out_bf16[idx] = __float2bfloat16(v);
    }
  }
}

template <class T, int BS, bool X2>
static void launch_t2(const QW& w, const ActQ8& x, int B, const GemvEpi& ep, cudaStream_t st) {
  if (ep.mode == EPI_SWIGLU_Q8) {
    constexpr int RW = 4, NW = 16;  // 64 rows = 32 gate + 32 up
    qgemv_kernel<T, BS, RW, NW, X2><<<w.N / 64, NW * 32, 0, st>>>(w, x, B, ep);
  } else {
    constexpr int RW = 2, NW = 4;
    int rows_per_cta = RW * NW;
    qgemv_kernel<T, BS, RW, NW, X2><<<(w.N + rows_per_cta - 1) / rows_per_cta, NW * 32, 0, st>>>(w, x, B, ep);
  }
}

template <class T, int BS>
static void launch_t(const QW& w, const ActQ8& x, int B, const GemvEpi& ep, cudaStream_t st) {
  if (x.ql)
    launch_t2<T, BS, true>(w, x, B, ep, st);
  else
    launch_t2<T, BS, false>(w, x, B, ep, st);
}

template <class T>
static void launch_bs(const QW& w, const ActQ8& x, int B, const GemvEpi& ep, cudaStream_t st) {
  if (B <= 1)
    launch_t<T, 1>(w, x, B, ep, st);
  else if (B <= 2)
    launch_t<T, 2>(w, x, B, ep, st);
  else if (B <= 4)
    launch_t<T, 4>(w, x, B, ep, st);
  else
    launch_t<T, 8>(w, x, B, ep, st);
}

int qgemv(const QW& w, const ActQ8& x, const __nv_bfloat16* xb, int ldxb, int B, const GemvEpi& ep,
          cudaStream_t st) {
  if (B < 1 || B > 8) return -1;
  if (w.type != W_BF16 && (w.K % 32)) return -2;
  if (ep.mode == EPI_SWIGLU_Q8 && (w.N % 64)) return -3;
  switch (w.type) {
    case W_Q4_0: launch_bs<T4Block<false>>(w, x, B, ep, st); break;
    case W_IQ4_NL: launch_bs<T4Block<true>>(w, x, B, ep, st); break;
    case W_Q8_0: launch_bs<TQ8_0>(w, x, B, ep, st); break;
    case W_Q4_K: if (w.K % 256) return -2; launch_bs<TK45<false>>(w, x, B, ep, st); break;
    case W_Q5_K: if (w.K % 256) return -2; launch_bs<TK45<true>>(w, x, B, ep, st); break;
    case W_Q6_K: if (w.K % 256) return -2; launch_bs<TQ6_K>(w, x, B, ep, st); break;
    case W_BF16: {
      if (ep.mode == EPI_SWIGLU_Q8) return -4;
      const __nv_bfloat16* W = reinterpret_cast<const __nv_bfloat16*>(w.p0);
      dim3 g((w.N + 3) / 4);
      if (B <= 1) bf16_gemv_kernel<1><<<g, 128, 0, st>>>(W, w.N, w.K, xb, ldxb, B, ep);
      else if (B <= 4) bf16_gemv_kernel<4><<<g, 128, 0, st>>>(W, w.N, w.K, xb, ldxb, B, ep);
      else bf16_gemv_kernel<8><<<g, 128, 0, st>>>(W, w.N, w.K, xb, ldxb, B, ep);
      break;
    }
    default: return -5;
  }
  return 0;
}

}  // namespace barq
