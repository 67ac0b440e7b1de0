// K12: fused sampler.  One CTA (512 threads) per sequence row of logits.
//
// Pipeline (the fixed order of the reference's sampler chain, sampling/src/chain.rs:11-112, and of
// ModelContext::sample, models/src/context.rs:418-516):
//   repetition / frequency / presence penalties -> grammar bitmask -> temperature ->
//   top-k -> top-p -> min-p -> sample (Philox4x32-10) | argmax when temperature <= 0.
//
// Top-k: a threshold is found by bisection on the logit value so that at least k tokens survive,
// the survivors (<= CAP) are sorted in shared memory and the first k kept; top-p and min-p then
// act on the sorted list, and the token is drawn by inverse CDF.  Without top-k, the nucleus
// threshold is found by bisection on probability mass and the token is drawn with the Gumbel-max
// trick over the survivors, which needs no sort and no candidate cap.
// Random numbers: Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3",
// SC 2011), keyed by the request seed and counted by (step, token index).
#include "common.cuh"
#include "pdl.cuh"
#include "launch.h"

namespace barq {

BARQ_DEV uint4 philox4x32_10(uint4 ctr, uint2 key) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    uint32_t hi0 = __umulhi(M0, ctr.x), lo0 = M0 * ctr.x;
    uint32_t hi1 = __umulhi(M1, ctr.z), lo1 = M1 * ctr.z;
    ctr = make_uint4(hi1 ^ ctr.y ^ key.x, lo1, hi0 ^ ctr.w ^ key.y, lo0);
    key.x += W0;
    key.y += W1;
  }
  return ctr;
}

BARQ_DEV float u01(uint32_t x) { return ((float)(x >> 8) + 0.5f) * (1.0f / 16777216.0f); }

constexpr int SNT = 512;
constexpr int CAP = 2048;

struct SampleShared {
  float red_f[SNT / 32];
  int red_i[SNT / 32];
  float cand_v[CAP];
  int cand_i[CAP];
  int n_cand;
};

BARQ_DEV float block_max(float v, SampleShared& sh) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) sh.red_f[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = threadIdx.x < SNT / 32 ? sh.red_f[threadIdx.x] : -INFINITY;
  if (threadIdx.x < 32) r = warp_max(r);
  __syncthreads();
  if (threadIdx.x == 0) sh.red_f[0] = r;
  __syncthreads();
  r = sh.red_f[0];
  __syncthreads();
  return r;
}

BARQ_DEV float block_sum(float v, SampleShared& sh) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) sh.red_f[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = threadIdx.x < SNT / 32 ? sh.red_f[threadIdx.x] : 0.f;
  if (threadIdx.x < 32) r = warp_sum(r);
  __syncthreads();
  if (threadIdx.x == 0) sh.red_f[0] = r;
  __syncthreads();
  r = sh.red_f[0];
  __syncthreads();
  return r;
}

// argmax with lowest-index tie break
BARQ_DEV void block_argmax(float& v, int& idx, SampleShared& sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, v, o);
    int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sh.red_f[threadIdx.x >> 5] = v;
    sh.red_i[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    v = threadIdx.x < SNT / 32 ? sh.red_f[threadIdx.x] : -INFINITY;
    idx = threadIdx.x < SNT / 32 ? sh.red_i[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, v, o);
      int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    if (threadIdx.x == 0) {
      sh.red_f[0] = v;
      sh.red_i[0] = idx;
    }
  }
  __syncthreads();
  v = sh.red_f[0];
  idx = sh.red_i[0];
  __syncthreads();
}

__global__ void __launch_bounds__(SNT) sample_kernel(SampleArgs a) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SampleShared& sh = *reinterpret_cast<SampleShared*>(smem_raw);
  const int b = blockIdx.x;
  float* row = const_cast<float*>(a.logits) + (size_t)b * a.ld;
  const int V = a.V;

  // 1) penalties over the token history (applied in place, once per distinct token)
  if (a.penalties && a.pen_counts_idx) {
    const float rep = a.penalties[b * 3 + 0], fq = a.penalties[b * 3 + 1], pr = a.penalties[b * 3 + 2];
    const int* hist = a.pen_counts_idx + (size_t)b * a.max_hist;
    for (int i = threadIdx.x; i < a.max_hist; i += SNT) {
      int t = hist[i];
      if (t < 0 || t >= V) continue;
      bool first = true;
      int cnt = 0;
      for (int j = 0; j < a.max_hist; ++j) {
        if (hist[j] == t) {
          if (j < i) first = false;
          ++cnt;
        }
      }
      if (!first) continue;
      float l = row[t];
      if (rep != 1.f) l = l > 0.f ? l / rep : l * rep;
      l -= (float)cnt * fq + pr;
      row[t] = l;
    }
    __syncthreads();
  }
  const uint32_t* mask = a.allow_mask ? a.allow_mask + (size_t)b * ((V + 31) / 32) : nullptr;
  auto logit = [&](int i) -> float {
    float l = row[i];
    if (mask && !((mask[i >> 5] >> (i & 31)) & 1u)) l = -INFINITY;
    return l;
  };

  const float temp = a.temperature ? a.temperature[b] : 0.f;
  // 2) greedy
  if (temp <= 0.f) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += SNT) {
      float l = logit(i);
      if (l > bv || (l == bv && i < bi)) {
        bv = l;
        bi = i;
      }
    }
    block_argmax(bv, bi, sh);
    if (threadIdx.x == 0) {
      a.out_ids[b] = bi < V ? bi : 0;
      if (a.out_logprob) a.out_logprob[b] = 0.f;
    }
    return;
  }
  const float it = 1.0f / temp;
  float mx = -INFINITY;
  for (int i = threadIdx.x; i < V; i += SNT) mx = fmaxf(mx, logit(i) * it);
  const float M = block_max(mx, sh);
  const int top_k = a.top_k ? a.top_k[b] : 0;
  const float top_p = a.top_p ? a.top_p[b] : 1.f;
  const float min_p = a.min_p ? a.min_p[b] : 0.f;
  const uint2 key = make_uint2((uint32_t)(a.seeds[b] & 0xffffffffu), (uint32_t)(a.seeds[b] >> 32));
  const uint32_t step = a.steps ? (uint32_t)a.steps[b] : 0u;

  if (top_k > 0) {
    const int k = min(top_k, CAP);
    // bisection: largest tau with count(l >= tau) >= k
    float lo = M - 80.f, hi = M;
    for (int iter = 0; iter < 24; ++iter) {
      float mid = 0.5f * (lo + hi);
      float c = 0.f;
      for (int i = threadIdx.x; i < V; i += SNT) c += (logit(i) * it >= mid) ? 1.f : 0.f;
      c = block_sum(c, sh);
      if (c >= (float)k) lo = mid; else hi = mid;
    }
    const float tau = lo;
    if (threadIdx.x == 0) sh.n_cand = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < V; i += SNT) {
      float l = logit(i) * it;
      if (l >= tau) {
        int s = atomicAdd(&sh.n_cand, 1);
        if (s < CAP) {
          sh.cand_v[s] = l;
          sh.cand_i[s] = i;
        }
      }
    }
    __syncthreads();
    const int n = min(sh.n_cand, CAP);
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    for (int i = n + threadIdx.x; i < np2; i += SNT) {
      sh.cand_v[i] = -INFINITY;
      sh.cand_i[i] = 0x7fffffff;
    }
    __syncthreads();
    // bitonic sort, descending by value (ties: lower index first)
    for (int size = 2; size <= np2; size <<= 1) {
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        for (int i = threadIdx.x; i < np2; i += SNT) {
          int j = i ^ stride;
          if (j > i) {
            bool desc = (i & size) == 0;
            float vi = sh.cand_v[i], vj = sh.cand_v[j];
            int ii = sh.cand_i[i], ij = sh.cand_i[j];
            bool i_first = vi > vj || (vi == vj && ii < ij);
            if (desc != i_first) {
              sh.cand_v[i] = vj;
              sh.cand_v[j] = vi;
              sh.cand_i[i] = ij;
              sh.cand_i[j] = ii;
            }
          }
        }
        __syncthreads();
      }
    }
    if (threadIdx.x == 0) {
      const int kk = min(k, n);
      float z = 0.f;
      for (int i = 0; i < kk; ++i) z += __expf(sh.cand_v[i] - M);
      // top-p and min-p on the sorted, renormalized top-k
      float cum = 0.f;
      int keep = kk;
      const float pmax = __expf(sh.cand_v[0] - M) / z;
      for (int i = 0; i < kk; ++i) {
        float p = __expf(sh.cand_v[i] - M) / z;
        if (min_p > 0.f && p < min_p * pmax) {
          keep = max(i, 1);
          break;
        }
        cum += p;
        if (cum >= top_p) {
          keep = i + 1;
          break;
        }
      }
      float z2 = 0.f;
      for (int i = 0; i < keep; ++i) z2 += __expf(sh.cand_v[i] - M);
      uint4 r = philox4x32_10(make_uint4(step, 0u, (uint32_t)b, 0x5a4d5u), key);
      float u = u01(r.x) * z2;
      int pick = keep - 1;
      float acc = 0.f;
      for (int i = 0; i < keep; ++i) {
        acc += __expf(sh.cand_v[i] - M);
        if (u <= acc) {
          pick = i;
          break;
        }
      }
      a.out_ids[b] = sh.cand_i[pick];
      if (a.out_logprob) a.out_logprob[b] = sh.cand_v[pick] - M - __logf(z2);
    }
    return;
  }
  // no top-k: nucleus threshold by bisection on mass, then Gumbel-max over survivors
  float tau = -INFINITY;
  float Z = 0.f;
  for (int i = threadIdx.x; i < V; i += SNT) Z += __expf(logit(i) * it - M);
  Z = block_sum(Z, sh);
  if (top_p < 1.f) {
    float lo = M - 80.f, hi = M;
    for (int iter = 0; iter < 24; ++iter) {
      float mid = 0.5f * (lo + hi);
      float s = 0.f;
      for (int i = threadIdx.x; i < V; i += SNT) {
        float l = logit(i) * it;
        if (l >= mid) s += __expf(l - M);
      }
      s = block_sum(s, sh);
      if (s >= top_p * Z) lo = mid; else hi = mid;
    }
    tau = lo;
  }
  if (min_p > 0.f) tau = fmaxf(tau, M + __logf(min_p));
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += SNT) {
    float l = logit(i) * it;
    if (l < tau || l == -INFINITY) continue;
    uint4 r = philox4x32_10(make_uint4(step, (uint32_t)i, (uint32_t)b, 0x6b5au), key);
    float g = l - __logf(-__logf(u01(r.x)));
    if (g > bv || (g == bv && i < bi)) {
      bv = g;
      bi = i;
    }
  }
  block_argmax(bv, bi, sh);
  if (threadIdx.x == 0) {
    int id = bi < V ? bi : 0;
    a.out_ids[b] = id;
    if (a.out_logprob) a.out_logprob[b] = row[id] * it - M - __logf(Z);
  }
}

int sample_tokens(const SampleArgs& a, cudaStream_t st) {
  if (a.B <= 0) return 0;
  size_t smem = sizeof(SampleShared);
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    attr_set = true;
  }
  launch_pdl(sample_kernel, dim3(a.B), dim3(SNT), smem, st, a);
  return 0;
}

}  // namespace barq

// ------------------------------------------------------------------------------------ K14
// Speculative-decoding verification on the device: one CTA, no host round trip until the result.
// ps: target distributions [k+1, V] (f32, rows for the k drafted positions and the bonus position);
// qs: draft distributions [k, V]; drafts: int64 [k].  Sampled: draft i is accepted while
// u_i < p_i(d_i) / q_i(d_i) (u_i from Philox keyed by seed, counter (step, i)); at the first
// rejection n the correction is drawn from norm(max(0, p_n - q_n)) (p_n itself if that is all
// zero), after k acceptances the bonus token from p_k -- the standard rejection rule, so the
// output follows the target distribution.  Greedy: accept while argmax(p_i) == d_i, then append
// argmax(p_n).  out: int32 [k + 2] = (n accepted, tokens[0..n]).
namespace barq {
namespace {
constexpr int VT = 1024;

BARQ_DEV float vblock_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  if (threadIdx.x < 32) {
    t = threadIdx.x < VT / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  t = red[32];
  __syncthreads();
  return t;
}

// argmax of a row (ties: lowest index)
BARQ_DEV int vblock_argmax(const float* row, int V, float* redv, int* redi) {
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += VT) {
    const float x = row[i];
    if (x > bv) {
      bv = x;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    redv[threadIdx.x >> 5] = bv;
    redi[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    bv = redv[threadIdx.x];
    bi = redi[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (threadIdx.x == 0) redi[32] = bi;
  }
  __syncthreads();
  const int r = redi[32];
  __syncthreads();
  return r;
}
}  // namespace

__global__ void __launch_bounds__(VT) spec_verify_kernel(const float* ps, const float* qs, const int64_t* drafts,
                                                         int k, int V, int greedy, uint64_t seed, uint32_t step,
                                                         int* out) {
  __shared__ float redv[33];
  __shared__ int redi[33];
  __shared__ float csum[VT];
  __shared__ int n_s;
  const uint2 key = make_uint2((uint32_t)(seed & 0xffffffffu), (uint32_t)(seed >> 32));
  if (threadIdx.x == 0) {
    int n = 0;
    if (!greedy) {
      for (; n < k; ++n) {
        const int64_t d = drafts[n];
        const float px = ps[(size_t)n * V + d], qx = fmaxf(qs[(size_t)n * V + d], 1e-20f);
        const uint4 r = philox4x32_10(make_uint4(step, (uint32_t)n, 0u, 0x7e57u), key);
        if (!(u01(r.x) < fminf(px / qx, 1.f))) break;
      }
    }
    n_s = n;
  }
  __syncthreads();
  int n = n_s;
  if (greedy) {  // accept while the target's argmax agrees with the draft
    for (n = 0; n < k; ++n)
      if (vblock_argmax(ps + (size_t)n * V, V, redv, redi) != (int)drafts[n]) break;
    const int tok = vblock_argmax(ps + (size_t)n * V, V, redv, redi);
    if (threadIdx.x == 0) {
      out[0] = n;
      for (int i = 0; i < n; ++i) out[1 + i] = (int)drafts[i];
      out[1 + n] = tok;
    }
    return;
  }
  // residual (or bonus) distribution r, sampled by inverse CDF over contiguous chunks
  const float* p = ps + (size_t)n * V;
  const float* q = n < k ? qs + (size_t)n * V : nullptr;
  const int per = (V + VT - 1) / VT, c0 = threadIdx.x * per, c1 = min(V, c0 + per);
  float s = 0.f;
  for (int i = c0; i < c1; ++i) s += q ? fmaxf(p[i] - q[i], 0.f) : p[i];
  float tot = vblock_sum(s, redv);
  bool use_p = q && !(tot > 0.f);  // p == q exactly: fall back to p
  if (use_p) {
    s = 0.f;
    for (int i = c0; i < c1; ++i) s += p[i];
    tot = vblock_sum(s, redv);
  }
  csum[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {  // exclusive prefix of the chunk sums (in place), then the target mass
    float run = 0.f;
    for (int i = 0; i < VT; ++i) {
      const float v = csum[i];
      csum[i] = run;
      run += v;
    }
    const uint4 r = philox4x32_10(make_uint4(step, (uint32_t)k, 1u, 0x7e57u), key);
    redv[32] = u01(r.x) * run;
  }
  __syncthreads();
  const float target = redv[32];
  if (threadIdx.x == 0) redi[32] = -1;
  __syncthreads();
  const float lo = csum[threadIdx.x];
  const float hi = threadIdx.x + 1 < VT ? csum[threadIdx.x + 1] : INFINITY;
  if (target >= lo && target < hi && c0 < c1) {
    float acc = lo;
    int pick = c1 - 1;
    for (int i = c0; i < c1; ++i) {
      acc += (q && !use_p) ? fmaxf(p[i] - q[i], 0.f) : p[i];
      if (target < acc) {
        pick = i;
        break;
      }
    }
    redi[32] = pick;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int tok = redi[32];
    if (tok < 0) tok = V - 1;  // the target fell past the last mass by rounding
    out[0] = n;
    for (int i = 0; i < n; ++i) out[1 + i] = (int)drafts[i];
    out[1 + n] = tok;
  }
}

int spec_verify(const float* ps, const float* qs, const int64_t* drafts, int k, int V, int greedy, uint64_t seed,
                uint32_t step, int* out, cudaStream_t st) {
  if (k < 0 || V <= 0) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(VT);
  cfg.stream = st;
  return cudaLaunchKernelEx(&cfg, spec_verify_kernel, ps, qs, drafts, k, V, greedy, seed, step, out) == cudaSuccess
             ? 0
             : -20;
}
}  // namespace barq
