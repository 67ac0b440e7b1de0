// K10: DeepSeek-V2 multi-head latent attention (MLA) over a paged latent cache.
//
// Parity: the reference declares MLA (models/src/deepseek.rs:55-78, advanced flash_mla.rs) but runs
// no attention for it; this is the absorbed form.  Each cached token is one 576-wide row: the
// RMS-normalized KV latent c (kv_lora_rank = 512) followed by the shared rotary key k_pe (64).  A
// query row holds, per head, q_lat = q_nope . W_UK (512, absorbed on the host side by a small GEMM)
// and the rotated q_pe (64).  Scores are q_lat . c + q_pe . k_pe, and the output stays in latent
// space (o_lat = softmax . c); o_lat . W_UV^T follows as another small GEMM.
//
//   mla_kv_write_kernel  per token: c = rmsnorm(kv_a[:512]) * w, k_pe = rope(kv_a[512:]) -> cache
//                        slot; the query's rope part is rotated in place.
//   mla_attn_kernel      grid (splits, query rows): all H heads of a row share each 16-token page,
//                        staged once in shared memory (rows padded by one float: conflict-free);
//                        thread (head, token) scores, per-head online softmax, thread (head, 32
//                        dims) accumulates; split partials + (max, sum) to scratch.
//   mla_merge_kernel     combines the splits of one (row, head).
#include "common.cuh"
#include "launch.h"
#include "pdl.cuh"

namespace barq {

namespace {
constexpr int kLat = 512, kRope = 64, kRow = kLat + kRope;  // 576
constexpr int kPage = 16;
constexpr int kMlaHeads = 16;
constexpr int kRowPad = kRow + 1;

template <typename TC>
__device__ __forceinline__ float ld_c(const TC* p) {
  if constexpr (std::is_same<TC, __half>::value)
    return __half2float(*p);
  else
    return __bfloat162float(*p);
}
template <typename TC>
__device__ __forceinline__ TC st_c(float v) {
  if constexpr (std::is_same<TC, __half>::value)
    return __float2half(v);
  else
    return __float2bfloat16(v);
}
}  // namespace

// One CTA per token, 256 threads.
template <typename TC>
__global__ void __launch_bounds__(256) mla_kv_write_kernel(MlaKvArgs a) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const float* kv = a.kv_a + (size_t)t * kRow;
  __shared__ float red[8];
  float ss = 0.f;
  for (int i = threadIdx.x; i < kLat; i += 256) ss += kv[i] * kv[i];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float rstd = rsqrtf(tot / (float)kLat + a.eps);
  const int pos = a.pos[t];
  TC* dst = reinterpret_cast<TC*>(a.cache) + (size_t)a.slots[t] * kRow;
  for (int i = threadIdx.x; i < kLat; i += 256) dst[i] = st_c<TC>(kv[i] * rstd * a.norm_w[i]);
  const float* cs = a.cos + (size_t)pos * (kRope / 2);
  const float* sn = a.sin + (size_t)pos * (kRope / 2);
  // rotary pairs: (2i, 2i+1) (normal) or (i, i + 32) (NeoX)
  if (threadIdx.x < kRope / 2) {
    const int i = threadIdx.x;
    const int i0 = a.neox ? i : 2 * i, i1 = a.neox ? i + kRope / 2 : 2 * i + 1;
    const float x0 = kv[kLat + i0], x1 = kv[kLat + i1];
    dst[kLat + i0] = st_c<TC>(x0 * cs[i] - x1 * sn[i]);
    dst[kLat + i1] = st_c<TC>(x0 * sn[i] + x1 * cs[i]);
  }
  // query rope part, in place: q [T, H, qdim], rope dims at [rope_off, rope_off + 64)
  for (int j = threadIdx.x; j < a.H * (kRope / 2); j += 256) {
    const int h = j / (kRope / 2), i = j % (kRope / 2);
    float* q = a.q + ((size_t)t * a.H + h) * a.qdim + a.rope_off;
    const int i0 = a.neox ? i : 2 * i, i1 = a.neox ? i + kRope / 2 : 2 * i + 1;
    const float x0 = q[i0], x1 = q[i1];
    q[i0] = x0 * cs[i] - x1 * sn[i];
    q[i1] = x0 * sn[i] + x1 * cs[i];
  }
}

// grid (splits, rows), 256 threads = 16 heads x 16 tokens of a page.
template <typename TC>
__global__ void __launch_bounds__(256) mla_attn_kernel(MlaAttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int split = blockIdx.x, row = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  extern __shared__ float sm[];
  float* qs = sm;                                // [16][kRowPad]
  float* cs = qs + kMlaHeads * kRowPad;          // [16][kRowPad]  page rows
  float* ps = cs + kPage * kRowPad;              // [16][16] probabilities
  float* alpha = ps + kMlaHeads * kPage;         // [16]
  const int seq = a.row_seq[row];
  const int len = a.row_len[row];  // visible cache tokens (causal)
  // query: q_lat (512) then q_pe (64) per head, f32
  for (int i = tid; i < kMlaHeads * kRow; i += 256) {
    const int h = i / kRow, d = i % kRow;
    const float v = d < kLat ? a.q_lat[((size_t)row * kMlaHeads + h) * kLat + d]
                             : a.q_pe[((size_t)row * kMlaHeads + h) * a.q_pe_stride + (d - kLat)];
    qs[h * kRowPad + d] = v * a.scale;
  }
  const int npages = (len + kPage - 1) / kPage;
  const int per = (npages + a.splits - 1) / a.splits;
  const int pb = split * per, pe = min(npages, pb + per);
  const int sh = tid >> 4, st = tid & 15;  // scoring: head sh, token st
  const int ah = tid >> 4, ad = tid & 15;  // accumulate: head ah, dims ad + 16 j
  float acc[kLat / 16];
#pragma unroll
  for (int j = 0; j < kLat / 16; ++j) acc[j] = 0.f;
  float m = -1e30f, l = 0.f;  // per head (held by every thread of the head's 16)
  __syncthreads();
  for (int pg = pb; pg < pe; ++pg) {
    const int blk = a.block_tables[(size_t)seq * a.max_blocks + pg];
    const TC* src = reinterpret_cast<const TC*>(a.cache) + (size_t)blk * kPage * kRow;
    for (int i = tid; i < kPage * kRow; i += 256) cs[(i / kRow) * kRowPad + (i % kRow)] = ld_c<TC>(src + i);
    __syncthreads();
    // scores
    float s = 0.f;
    const float* qh = qs + sh * kRowPad;
    const float* ct = cs + st * kRowPad;
#pragma unroll 8
    for (int d = 0; d < kRow; ++d) s = fmaf(qh[d], ct[d], s);
    const bool valid = pg * kPage + st < len;
    s = valid ? s : -INFINITY;
    // online softmax over the 16 tokens of head sh (a half-warp)
    float mx = s;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float m_new = fmaxf(m, mx);
    const float p = valid ? __expf(s - m_new) : 0.f;
    float psum = p;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    const float al = __expf(m - m_new);
    l = l * al + psum;
    m = m_new;
    ps[sh * kPage + st] = p;
    if (st == 0) alpha[sh] = al;
    __syncthreads();
    // accumulate (thread head ah == sh: the same per-head state)
    const float alh = alpha[ah];
#pragma unroll
    for (int j = 0; j < kLat / 16; ++j) {
      const int d = ad + 16 * j;
      float v = acc[j] * alh;
#pragma unroll
      for (int t = 0; t < kPage; ++t) v = fmaf(ps[ah * kPage + t], cs[t * kRowPad + d], v);
      acc[j] = v;
    }
    __syncthreads();
  }
  // partials
  const size_t pbase = ((size_t)row * a.splits + split) * kMlaHeads + ah;
#pragma unroll
  for (int j = 0; j < kLat / 16; ++j) a.part_acc[pbase * kLat + ad + 16 * j] = acc[j];
  if (ad == 0) a.part_ml[pbase] = make_float2(m, l);
  (void)warp;
  (void)lane;
}

// grid (heads, rows), 256 threads; o_lat [rows, H, 512] f32.
__global__ void __launch_bounds__(256) mla_merge_kernel(MlaAttnArgs a) {
  pdl_wait();
  pdl_trigger();
  const int h = blockIdx.x, row = blockIdx.y;
  float M = -1e30f;
  for (int s = 0; s < a.splits; ++s) M = fmaxf(M, a.part_ml[((size_t)row * a.splits + s) * kMlaHeads + h].x);
  float L = 0.f;
  for (int s = 0; s < a.splits; ++s) {
    const float2 ml = a.part_ml[((size_t)row * a.splits + s) * kMlaHeads + h];
    L += ml.y * __expf(ml.x - M);
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  for (int d = threadIdx.x; d < kLat; d += 256) {
    float o = 0.f;
    for (int s = 0; s < a.splits; ++s) {
      const size_t pb = ((size_t)row * a.splits + s) * kMlaHeads + h;
      o += a.part_acc[pb * kLat + d] * __expf(a.part_ml[pb].x - M);
    }
    a.o_lat[((size_t)row * kMlaHeads + h) * kLat + d] = o * inv;
  }
}

int mla_kv_write(const MlaKvArgs& a, int cache_is_bf16, cudaStream_t st) {
  if (a.T <= 0) return 0;
  cudaError_t e = cache_is_bf16 ? launch_pdl(mla_kv_write_kernel<__nv_bfloat16>, dim3(a.T), dim3(256), 0, st, a)
                                : launch_pdl(mla_kv_write_kernel<__half>, dim3(a.T), dim3(256), 0, st, a);
  return e == cudaSuccess ? 0 : -20;
}

size_t mla_attn_scratch_floats(int rows, int splits) {
  return (size_t)rows * splits * kMlaHeads * (kLat + 2);
}

int mla_attention(const MlaAttnArgs& a, int cache_is_bf16, cudaStream_t st) {
  if (a.H != kMlaHeads) return -1;
  if (a.splits < 1 || a.splits > 64) return -2;
  if (a.rows <= 0) return 0;
  const int smem = (2 * kMlaHeads * kRowPad + kMlaHeads * kPage + kMlaHeads) * (int)sizeof(float);
  auto k16 = mla_attn_kernel<__half>;
  auto kb16 = mla_attn_kernel<__nv_bfloat16>;
  cudaFuncSetAttribute(k16, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaFuncSetAttribute(kb16, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaError_t e = cache_is_bf16 ? launch_pdl(kb16, dim3(a.splits, a.rows), dim3(256), (size_t)smem, st, a)
                                : launch_pdl(k16, dim3(a.splits, a.rows), dim3(256), (size_t)smem, st, a);
  if (e == cudaSuccess) e = launch_pdl(mla_merge_kernel, dim3(kMlaHeads, a.rows), dim3(256), 0, st, a);
  return e == cudaSuccess ? 0 : -20;
}

}  // namespace barq
