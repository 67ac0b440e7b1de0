// K8: paged flash-decode attention (one new query token per sequence), GQA-packed, split-KV.
//
// The reference has no attention kernel at all: FlashAttention::forward* returns Unsupported
// (backend/src/cuda_flash_attn.rs:165-359) and the CPU path loops over heads and query rows
// (models/src/transformer.rs:301-374).
//
// Grid (splits, Hkv, B), 4 warps per CTA.  All G = H/Hkv query heads of a KV head share one CTA,
// so every K/V page (16 tokens x D, fp16/bf16) is read from HBM once per step.  A warp takes one
// page at a time: for QK^T two lanes share a token (each half of D in interleaved 16-byte chunks,
// which keeps both the page loads coalesced and the shared-memory q reads conflict-free); for PV
// each lane owns D/32 output dims and receives the probabilities by shuffle.  Each warp keeps an
// online-softmax state; the CTA merges its 4 warps and writes an unnormalized partial per split.
// The splits are then merged (normalized, written as bf16/fp16 and as the int8 q8 activation of
// the output projection) by the last split CTA of each (sequence, KV head) to arrive -- a counter
// per (b, kv head) finds it, and it resets the counter -- or, without counters, by a second kernel.
#include "common.cuh"
#include "pdl.cuh"
#include "launch.h"

namespace barq {

// 8 consecutive K elements (one "chunk") of a row as floats: 16-byte loads for 2-byte types, 8-byte
// loads for fp8.
template <typename TC>
BARQ_DEV void load_k8(const TC* row, int chunk, float* f);
template <typename TC> BARQ_DEV void cvt8(const int4& raw, float* f);
template <> BARQ_DEV void cvt8<__half>(const int4& raw, float* f) {
  const __half2* h = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 v = __half22float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}
template <> BARQ_DEV void cvt8<__nv_bfloat16>(const int4& raw, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&raw);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 v = __bfloat1622float2(h[i]);
    f[2 * i] = v.x;
    f[2 * i + 1] = v.y;
  }
}

template <> BARQ_DEV void load_k8<__half>(const __half* row, int chunk, float* f) {
  cvt8<__half>(__ldg(reinterpret_cast<const int4*>(row) + chunk), f);
}
template <> BARQ_DEV void load_k8<__nv_bfloat16>(const __nv_bfloat16* row, int chunk, float* f) {
  cvt8<__nv_bfloat16>(__ldg(reinterpret_cast<const int4*>(row) + chunk), f);
}
template <> BARQ_DEV void load_k8<__nv_fp8_e4m3>(const __nv_fp8_e4m3* row, int chunk, float* f) {
  const uint2 raw = __ldg(reinterpret_cast<const uint2*>(row) + chunk);
  const __nv_fp8_e4m3* e = reinterpret_cast<const __nv_fp8_e4m3*>(&raw);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = static_cast<float>(e[i]);
}

constexpr int kBS = 16;  // tokens per KV page

// This lane's DPL consecutive V elements of one token, kept packed in registers until used.
template <typename TC, int DPL>
struct VRow {
  static constexpr int BYTES = DPL * (int)sizeof(TC);
  using R = typename std::conditional<BYTES == 8, uint2,
                                      typename std::conditional<BYTES == 4, uint32_t, unsigned short>::type>::type;
  R r;
  BARQ_DEV void load(const TC* p) { r = __ldg(reinterpret_cast<const R*>(p)); }
  BARQ_DEV void cvt(float* f) const {
    const TC* e = reinterpret_cast<const TC*>(&r);
#pragma unroll
    for (int i = 0; i < DPL; ++i) f[i] = to_f(e[i]);
  }
};

template <typename TC, int D, int G>
__global__ void __launch_bounds__(128) decode_attn_kernel(DecodeAttnArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int NW = 4;
  constexpr int CH = D / 8;        // 16-byte chunks per K row
  constexpr int CPH = CH / 2;      // chunks per half-lane
  constexpr int DPL = D / 32;      // output dims per lane
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float LOG2E = 1.4426950408889634f;

  __shared__ float q_s[G][D];
  __shared__ float m_s[NW][G], l_s[NW][G];
  __shared__ float acc_s[NW][G][D];

  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    int g = i / D, d = i % D;
    q_s[g][d] = __bfloat162float(a.q[((size_t)b * a.H + kvh * G + g) * D + d]) * a.scale * LOG2E;
  }
  __syncthreads();

  const int seq_len = a.seq_lens[b];
  const int first_tok = a.window > 0 ? max(0, seq_len - a.window) : 0;
  const int blk0 = first_tok / kBS;
  const int nblk = (seq_len + kBS - 1) / kBS - blk0;
  const int per = (nblk + a.splits - 1) / a.splits;
  const int sb = blk0 + split * per;
  const int se = min(blk0 + nblk, sb + per);

  float m[G], l[G], acc[G][DPL];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    m[g] = -1e30f;
    l[g] = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc[g][j] = 0.f;
  }
  const int tok = lane >> 1, half = lane & 1;
  const int* bt = a.block_tables + (size_t)b * a.max_blocks;
  const TC* kc = reinterpret_cast<const TC*>(a.kcache);
  const TC* vc = reinterpret_cast<const TC*>(a.vcache);

  for (int blk = sb + warp; blk < se; blk += NW) {
    const int phys = bt[blk];
    const size_t page = ((size_t)phys * a.Hkv + kvh) * kBS;
    const TC* krow = kc + (page + tok) * D;
    // The page's V rows are loaded together with K (they do not depend on the scores), so a page
    // costs one DRAM round trip instead of two.
    const TC* vpage = vc + page * D;
    VRow<TC, DPL> vr[kBS];
#pragma unroll
    for (int t = 0; t < kBS; ++t) vr[t].load(vpage + (size_t)t * D + lane * DPL);
    float s[G];
#pragma unroll
    for (int g = 0; g < G; ++g) s[g] = 0.f;
#pragma unroll
    for (int c = 0; c < CPH; ++c) {
      const int chunk = 2 * c + half;
      float kf[8];
      load_k8<TC>(krow, chunk, kf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4* qv = reinterpret_cast<const float4*>(&q_s[g][chunk * 8]);
        float4 q0 = qv[0], q1 = qv[1];
        s[g] += q0.x * kf[0] + q0.y * kf[1] + q0.z * kf[2] + q0.w * kf[3] + q1.x * kf[4] + q1.y * kf[5] +
                q1.z * kf[6] + q1.w * kf[7];
      }
    }
    const int tpos = blk * kBS + tok;
    const bool valid = tpos < seq_len && tpos >= first_tok;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      s[g] += __shfl_xor_sync(0xffffffffu, s[g], 1);
      if (!valid) s[g] = -INFINITY;
    }
    // online softmax update (scores already in log2 units)
    float p[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      float mx = warp_max(s[g]);
      float mn = fmaxf(m[g], mx);
      float corr = exp2f(m[g] - mn);
      p[g] = exp2f(s[g] - mn);
      float ps = warp_sum(half == 0 ? p[g] : 0.f);
      l[g] = l[g] * corr + ps;
      m[g] = mn;
#pragma unroll
      for (int j = 0; j < DPL; ++j) acc[g][j] *= corr;
    }
#pragma unroll
    for (int t = 0; t < kBS; ++t) {
      float vf[DPL];
      vr[t].cvt(vf);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float pt = __shfl_sync(0xffffffffu, p[g], 2 * t);
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[g][j] += pt * vf[j];
      }
    }
  }
  // merge the 4 warps of this CTA
  if (lane == 0) {
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m_s[warp][g] = m[g];
      l_s[warp][g] = l[g];
    }
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int j = 0; j < DPL; ++j) acc_s[warp][g][lane * DPL + j] = acc[g][j];
  __syncthreads();
  const size_t pbase = (((size_t)b * a.Hkv + kvh) * a.splits + split) * G;
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {
    int g = i / D, d = i % D;
    float M = -1e30f;
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, m_s[w][g]);
    float A = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < NW; ++w) {
      float f = exp2f(m_s[w][g] - M);
      A += acc_s[w][g][d] * f;
      L += l_s[w][g] * f;
    }
    a.part_acc[(pbase + g) * D + d] = A;
    if (d == 0) a.part_ml[pbase + g] = make_float2(M, L);
  }
  if (!a.counters) return;
  // ---- in-kernel merge by the last split CTA of this (b, kv head)
  __shared__ int last_s;
  __threadfence();  // this CTA's partial before its arrival
  __syncthreads();
  int* cnt = a.counters + (size_t)b * a.Hkv + kvh;
  if (threadIdx.x == 0) last_s = atomicAdd(cnt, 1) == a.splits - 1;
  __syncthreads();
  if (!last_s) return;
  __threadfence();  // every other split's partial (they fenced before arriving) before the reads
  const size_t sbase = ((size_t)b * a.Hkv + kvh) * a.splits;
  // per-split weights exp2(m_s - M) and 1 / L once per head, then one pass over the accumulators
  __shared__ float2 ml_x[G][64];
  __shared__ float fw_s[G][64], inv_s[G];
  for (int i = threadIdx.x; i < G * a.splits; i += blockDim.x) {
    const int g = i / a.splits, sp = i - g * a.splits;
    ml_x[g][sp] = __ldcg(&a.part_ml[(sbase + sp) * G + g]);
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    float M = -1e30f, L = 0.f;
    for (int sp = 0; sp < a.splits; ++sp) M = fmaxf(M, ml_x[g][sp].x);
    for (int sp = 0; sp < a.splits; ++sp) {
      const float f = exp2f(ml_x[g][sp].x - M);
      fw_s[g][sp] = f;
      L += ml_x[g][sp].y * f;
    }
    inv_s[g] = L > 0.f ? 1.f / L : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * D; i += blockDim.x) {  // warp-uniform: G * D is a multiple of 32
    const int g = i / D, d = i % D;
    const float* pa = a.part_acc + (sbase * G + g) * D + d;
    float A = 0.f;
#pragma unroll 8
    for (int sp = 0; sp < a.splits; ++sp) A += __ldcg(pa + (size_t)sp * G * D) * fw_s[g][sp];
    const float o = A * inv_s[g];
    const size_t oi = (size_t)b * a.H * D + (size_t)(kvh * G + g) * D + d;
    store_act(a.out, oi, o, a.out_f16);
    if (a.out_q.q) act_store32(a.out_q, o, oi, oi / 32, d & 31);
  }
  if (threadIdx.x == 0) *cnt = 0;  // ready for the next call / graph replay
}

// One CTA per (head, batch row); D threads.
template <int D>
__global__ void __launch_bounds__(D) decode_merge_kernel(DecodeAttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int G = a.H / a.Hkv, kvh = h / G, g = h % G;
  const size_t base = ((size_t)b * a.Hkv + kvh) * a.splits;
  // (max, sum) of every split staged in shared memory with one parallel load, then a single pass
  // over the partial accumulators with independent (unrolled) loads.
  __shared__ float2 ml_s[64];
  __shared__ float M_s;
  for (int s = d; s < a.splits; s += D) ml_s[s] = a.part_ml[(base + s) * G + g];
  __syncthreads();
  if (d < 32) {
    float mx = -1e30f;
    for (int s = d; s < a.splits; s += 32) mx = fmaxf(mx, ml_s[s].x);
    mx = warp_max(mx);
    if (d == 0) M_s = mx;
  }
  __syncthreads();
  const float M = M_s;
  float A = 0.f, L = 0.f;
#pragma unroll 8
  for (int s = 0; s < a.splits; ++s) {
    const float2 ml = ml_s[s];
    const float f = exp2f(ml.x - M);
    L += ml.y * f;
    A += a.part_acc[((base + s) * G + g) * D + d] * f;
  }
  float o = L > 0.f ? A / L : 0.f;
  const size_t oi = (size_t)b * a.H * D + (size_t)h * D + d;
  store_act(a.out, oi, o, a.out_f16);
  if (a.out_q.q) act_store32(a.out_q, o, oi, oi / 32, d & 31);
}

size_t decode_attention_scratch_floats(int B, int H, int Hkv, int D, int splits) {
  return (size_t)B * H * splits * D + (size_t)B * H * splits * 2;
}

template <typename TC, int D>
static int launch_g(const DecodeAttnArgs& a, cudaStream_t st) {
  const int G = a.H / a.Hkv;
  dim3 grid(a.splits, a.Hkv, a.B);
  cudaError_t e;
  switch (G) {
    case 1: e = launch_pdl(decode_attn_kernel<TC, D, 1>, grid, dim3(128), 0, st, a); break;
    case 2: e = launch_pdl(decode_attn_kernel<TC, D, 2>, grid, dim3(128), 0, st, a); break;
    case 4: e = launch_pdl(decode_attn_kernel<TC, D, 4>, grid, dim3(128), 0, st, a); break;
    case 8: e = launch_pdl(decode_attn_kernel<TC, D, 8>, grid, dim3(128), 0, st, a); break;
    default: return -3;
  }
  if (e != cudaSuccess) return -20;
  if (!a.counters && launch_pdl(decode_merge_kernel<D>, dim3(a.H, a.B), dim3(D), 0, st, a) != cudaSuccess) return -20;
  return 0;
}

int decode_attention(const DecodeAttnArgs& a, cudaStream_t st) {
  if (a.block_size != kBS) return -1;
  if (a.splits < 1 || a.splits > 64) return -5;
  if (a.H % a.Hkv) return -2;
  if (a.B <= 0) return 0;
  if (a.D == 128)
    return a.cache_type == kCacheBF16  ? launch_g<__nv_bfloat16, 128>(a, st)
           : a.cache_type == kCacheFP8 ? launch_g<__nv_fp8_e4m3, 128>(a, st)
                                       : launch_g<__half, 128>(a, st);
  if (a.D == 64)
    return a.cache_type == kCacheBF16  ? launch_g<__nv_bfloat16, 64>(a, st)
           : a.cache_type == kCacheFP8 ? launch_g<__nv_fp8_e4m3, 64>(a, st)
                                       : launch_g<__half, 64>(a, st);
  return -4;
}

}  // namespace barq
