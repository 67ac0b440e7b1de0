// K11 pieces and small fused ops: residual-add + RMSNorm (-> bf16 / int8 q8), activation
// quantization, SwiGLU, RoPE + paged KV write, embedding gather, row dequantization.
//
// Parity: the reference's rms_norm / rope / SwiGLU run as separate f32 CPU loops
// (models/src/transformer.rs:148-172, 378-408, 514-568); here they are fused into the producers
// and consumers of each GEMV/GEMM so the residual stream is touched once per sub-layer.
#include <cstdlib>

#include "common.cuh"
#include "launch.h"
#include "pdl.cuh"
#include "qweight.cuh"

namespace barq {

// One CTA per token row, 1024 threads (32 warps), so a decode row of 4096 values is 4 groups of
// 32 per warp: the per-group quantization reductions run in parallel instead of in series.
constexpr int kNormThreads = 1024;
__global__ void __launch_bounds__(kNormThreads) rmsnorm_kernel(float* __restrict__ x, const float* __restrict__ add,
                                                      const float* __restrict__ w, float eps, int H,
                                                      void* __restrict__ ob, int ob_f16, ActOut oq) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  float* xr = x + (size_t)t * H;
  const float* ar = add ? add + (size_t)t * H : nullptr;
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += kNormThreads) {
    float v = xr[i];
    if (ar) {
      v += ar[i];
      xr[i] = v;
    }
    ss += v * v;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = red[threadIdx.x];
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / (float)H + eps);
  // Each warp walks 32-value groups so the q8 quantization of a group happens inside one warp.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ngroups = (H + 31) / 32;
  for (int g = warp; g < ngroups; g += kNormThreads / 32) {
    int i = g * 32 + lane;
    float v = i < H ? xr[i] * r * w[i] : 0.f;
    if (ob && i < H) store_act(ob, (size_t)t * H + i, v, ob_f16);
    if (oq.q) act_store32(oq, v, (size_t)t * H + i, (size_t)t * (H / 32) + g, lane);
  }
}

int rmsnorm(float* x, const float* add, const float* w, float eps, int T, int H, void* out_act, int out_f16,
            ActOut out_q, cudaStream_t st) {
  if (out_q.q && (H % 32)) return -1;
  if (T <= 0) return 0;
  return launch_pdl(rmsnorm_kernel, dim3(T), dim3(kNormThreads), 0, st, x, add, w, eps, H, out_act, out_f16, out_q) ==
                 cudaSuccess
             ? 0
             : -20;
}

template <typename T>
__global__ void quant_q8_kernel(const T* __restrict__ x, int H, int ldx, ActOut oq) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.y;
  const int g = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (g * 32 >= H) return;
  float v = to_f(x[(size_t)t * ldx + g * 32 + lane]);
  act_store32(oq, v, (size_t)t * H + g * 32 + lane, (size_t)t * (H / 32) + g, lane);
}

int quantize_q8(const void* x, int x_is_bf16, int T, int H, int ldx, ActOut out_q, cudaStream_t st) {
  if (H % 32) return -1;
  if (T <= 0) return 0;
  dim3 g((H / 32 + 7) / 8, T);
  const cudaError_t e =
      x_is_bf16 ? launch_pdl(quant_q8_kernel<__nv_bfloat16>, g, dim3(256), 0, st, (const __nv_bfloat16*)x, H, ldx, out_q)
                : launch_pdl(quant_q8_kernel<float>, g, dim3(256), 0, st, (const float*)x, H, ldx, out_q);
  return e == cudaSuccess ? 0 : -20;
}

template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ in, int F, int ld, void* __restrict__ ob, int ob_f16,
                              ActOut oq) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.y;
  const int lane = threadIdx.x & 31;
  const int g = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int i = g * 32 + lane;
  if (g * 32 >= F) return;
  float h = 0.f;
  if (i < F) h = silu(to_f(in[(size_t)t * ld + i])) * to_f(in[(size_t)t * ld + F + i]);
  if (ob && i < F) store_act(ob, (size_t)t * F + i, h, ob_f16);
  if (oq.q) act_store32(oq, h, (size_t)t * F + i, (size_t)t * (F / 32) + g, lane);
}

int swiglu(const void* in, int in_is_bf16, int T, int F, int ld_in, void* out_act, int out_f16, ActOut out_q,
           cudaStream_t st) {
  if (out_q.q && (F % 32)) return -1;
  if (T <= 0) return 0;
  dim3 g(((F + 31) / 32 + 7) / 8, T);
  const cudaError_t e =
      in_is_bf16 ? launch_pdl(swiglu_kernel<__nv_bfloat16>, g, dim3(256), 0, st, (const __nv_bfloat16*)in, F, ld_in,
                              out_act, out_f16, out_q)
                 : launch_pdl(swiglu_kernel<float>, g, dim3(256), 0, st, (const float*)in, F, ld_in, out_act, out_f16,
                              out_q);
  return e == cudaSuccess ? 0 : -20;
}

// ------------------------------------------------------------------------------ RoPE + KV write
// One CTA per token, one warp per head (q heads first, then k heads, then v heads).
template <typename TIN, typename TC>
__global__ void __launch_bounds__(256) rope_kv_kernel(RopeKVArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nh = a.H + 2 * a.Hkv;
  const TIN* row = reinterpret_cast<const TIN*>(a.qkv) + (size_t)t * a.ld_qkv;
  const int pos = a.pos[t];
  const int64_t slot = a.slots ? a.slots[t] : -1;
  const int D = a.D, half = a.rot / 2;
  const float* cs = a.cos_t + (size_t)pos * half;
  const float* sn = a.sin_t + (size_t)pos * half;
  for (int h = warp + blockIdx.y * 8; h < nh; h += 8 * gridDim.y) {
    const TIN* src = row + (size_t)h * D;
    const bool is_q = h < a.H, is_k = !is_q && h < a.H + a.Hkv;
    // Load the head (D <= 256) into registers: lane owns elements lane + 32*j.
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      int i = lane + 32 * j;
      v[j] = i < D ? to_f(src[i]) : 0.f;
    }
    const float* nw = is_q ? a.q_norm : (is_k ? a.k_norm : nullptr);
    if (nw) {
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[j] * v[j];
      ss = warp_sum(ss);
      float r = rsqrtf(ss / D + a.norm_eps);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        int i = lane + 32 * j;
        if (i < D) v[j] = v[j] * r * nw[i];
      }
    }
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = v[j];
    if (is_q || is_k) {
      // Rotate pairs: neox (i, i+half) or normal (2i, 2i+1); partner values fetched by shuffle
      // through a shared staging row.
      __shared__ float stage[8][256];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        int i = lane + 32 * j;
        if (i < D) stage[warp][i] = v[j];
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        int i = lane + 32 * j;
        if (i < a.rot) {
          int pi, fi;
          float sign;
          if (a.neox) {
            fi = i < half ? i : i - half;
            pi = i < half ? i + half : i - half;
            sign = i < half ? -1.f : 1.f;
          } else {
            fi = i >> 1;
            pi = i ^ 1;
            sign = (i & 1) ? 1.f : -1.f;
          }
          float c = cs[fi], s = sn[fi];
          o[j] = v[j] * c + sign * stage[warp][pi] * s;
        }
      }
      __syncwarp();
    }
    if (is_q) {
      __nv_bfloat16* dst = a.q_out + ((size_t)t * a.H + h) * D;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        int i = lane + 32 * j;
        if (i < D) dst[i] = __float2bfloat16(o[j]);
      }
    } else if (slot >= 0) {
      const int kvh = is_k ? h - a.H : h - a.H - a.Hkv;
      const int64_t blk = slot / a.block_size, off = slot % a.block_size;
      TC* cache = reinterpret_cast<TC*>(is_k ? a.kcache : a.vcache);
      const size_t ri = ((size_t)blk * a.Hkv + kvh) * a.block_size + off;  // stored row
      TC* dst = cache + ri * D;
      float* sc = is_k ? a.kscale : a.vscale;
      float inv = 1.f;
      if (sc) {  // scaled fp8: the row's largest magnitude maps to e4m3's 448
        float mx = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (lane + 32 * j < D) mx = fmaxf(mx, fabsf(o[j]));
        mx = warp_max(mx);
        const float s = mx > 0.f ? mx / 448.f : 1.f;
        inv = 1.f / s;
        if (lane == 0) sc[ri] = s;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        int i = lane + 32 * j;
        if (i < D) dst[i] = from_f<TC>(o[j] * inv);
      }
    }
  }
}

int rope_kv_write(const RopeKVArgs& a, cudaStream_t st) {
  if (a.D > 256 || a.rot > a.D || (a.rot & 1)) return -1;
  if (a.T <= 0) return 0;
  const int nh = a.H + 2 * a.Hkv;
  dim3 g(a.T, (nh + 7) / 8 > 4 ? 4 : (nh + 7) / 8);
  cudaError_t e;
  if (a.qkv_is_bf16) {
    if (a.cache_type == kCacheBF16) e = launch_pdl(rope_kv_kernel<__nv_bfloat16, __nv_bfloat16>, g, dim3(256), 0, st, a);
    else if (a.cache_type == kCacheFP8) e = launch_pdl(rope_kv_kernel<__nv_bfloat16, __nv_fp8_e4m3>, g, dim3(256), 0, st, a);
    else e = launch_pdl(rope_kv_kernel<__nv_bfloat16, __half>, g, dim3(256), 0, st, a);
  } else {
    if (a.cache_type == kCacheBF16) e = launch_pdl(rope_kv_kernel<float, __nv_bfloat16>, g, dim3(256), 0, st, a);
    else if (a.cache_type == kCacheFP8) e = launch_pdl(rope_kv_kernel<float, __nv_fp8_e4m3>, g, dim3(256), 0, st, a);
    else e = launch_pdl(rope_kv_kernel<float, __half>, g, dim3(256), 0, st, a);
  }
  return e == cudaSuccess ? 0 : -20;
}

}  // namespace barq

namespace barq {
static int g_pdl_mode = -1;  // -1: from BARQ_PDL (default on), 0: off, 1: on
bool pdl_enabled() {
  static const bool env_on = [] {
    const char* e = getenv("BARQ_PDL");
    return !(e && e[0] == '0');
  }();
  return env_on && g_pdl_mode != 0;
}
void set_pdl_mode(int mode) { g_pdl_mode = mode; }
}  // namespace barq
