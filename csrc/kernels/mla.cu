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
//   mla_attn_mma_kernel  the same work on the tensor cores (selected with impl = 1); see below.
//   mla_merge_kernel     combines the splits of one (row, head).
#include "common.cuh"
#include "launch.h"
#include "mma_sync.cuh"
#include "pdl.cuh"
#include "tc_common.cuh"

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

// ---------------------------------------------------------------------------------------------
// Tensor-core MLA decode attention.  grid (splits, rows), 4 compute warps + 1 copy warp.
//
// The 16 heads of a query row are exactly the 16 rows of an mma.m16n8k16 tile, and every head
// reads the same latent row per token, so one 16-token page (16 x 576, bf16 / fp16) is one B
// operand for all heads.  The copy warp streams the CTA's pages with cp.async into a 4-slot ring
// (rows padded to 584 elements: conflict-free ldmatrix) and signals per slot on an mbarrier.
// A 576-deep score row and a 512-wide output row are too wide for one warp's registers, so the
// compute warps split the dimensions and meet once per page:
//   * warp w holds the query fragments of dims [144 w, 144 w + 144) and computes that slice's
//     partial scores S_w = Q_w C_w^T (16 heads x 16 tokens, 18 MMAs);
//   * the partials go through shared memory (double-buffered by page parity) and a named barrier
//     over the 128 compute threads; every warp adds the four in warp order, so all four hold the
//     identical S, run the identical online softmax (log2 domain) and hold identical P;
//   * warp w accumulates O[:, 128 w : 128 w + 128] += P C[:, 128 w : 128 w + 128] (16 MMAs) and
//     releases the slot (the empty barrier counts the four compute warps).
// Each warp writes its 128 dims of the unnormalised split partial; (m, l) are stored in natural-log
// units so that mla_merge_kernel combines these partials unchanged.
// Waits are bounded (tc::mbar_wait); a warp whose wait fails marks the page's stop flag before the
// named barrier and every compute warp reads it after the barrier, so they leave the loop together.
constexpr int kMlaRing = 4;
constexpr int kMlaThreads = 160;
constexpr int kMlaLd = kRow + 8;  // 584 elements per shared-memory row

template <typename TC>
struct MlaRing {
  static constexpr int PAGE = kPage * kMlaLd * (int)sizeof(TC);  // one 16-token page
  static constexpr int QOFF = kMlaRing * PAGE;                    // the 16 query heads
  static constexpr int XOFF = QOFF + 16 * kMlaLd * (int)sizeof(TC);
  static constexpr int XBYTES = 2 * 4 * 16 * 16 * (int)sizeof(float);  // [parity][warp][16][16] partial S
  static constexpr int BYTES = XOFF + XBYTES;
  static_assert(PAGE % 16 == 0 && QOFF % 16 == 0 && XOFF % 16 == 0, "16-byte aligned regions");
};

template <typename TC>
__global__ void __launch_bounds__(kMlaThreads) mla_attn_mma_kernel(MlaAttnArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int NW = 4;
  constexpr int KSW = kRow / 16 / NW;  // 9 score k-steps per warp
  constexpr int NDW = kLat / 8 / NW;   // 16 output n-blocks per warp
  static_assert(KSW * 16 * NW == kRow && NDW * 8 * NW == kLat && NDW % 2 == 0, "dimension split");
  using R = MlaRing<TC>;
  const int split = blockIdx.x, row = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr float kLog2e = 1.4426950408889634f, kLn2 = 0.6931471805599453f;

  extern __shared__ __align__(128) uint8_t ring[];
  TC* sQ = reinterpret_cast<TC*>(ring + R::QOFF);
  float* sx = reinterpret_cast<float*>(ring + R::XOFF);
  __shared__ __align__(8) uint64_t full[kMlaRing], empty[kMlaRing];
  __shared__ int err_s, stop_s[2];
  if (threadIdx.x == 0) {
    err_s = 0;
    stop_s[0] = stop_s[1] = 0;
    for (int i = 0; i < kMlaRing; ++i) {
      tc::mbar_init(&full[i], 32);  // one arrival per copy-warp lane
      tc::mbar_init(&empty[i], NW);  // one per compute warp
    }
    tc::fence_mbar_init();
  }
  // the query heads as MMA rows, pre-scaled by the softmax scale
  for (int i = threadIdx.x; i < kMlaHeads * kRow; i += blockDim.x) {
    const int h = i / kRow, d = i % kRow;
    const float v = d < kLat ? a.q_lat[((size_t)row * kMlaHeads + h) * kLat + d]
                             : a.q_pe[((size_t)row * kMlaHeads + h) * a.q_pe_stride + (d - kLat)];
    sQ[h * kMlaLd + d] = from_f<TC>(v * a.scale);
  }
  __syncthreads();
  volatile int* err = &err_s;
  volatile int* stop = stop_s;

  const int seq = a.row_seq[row];
  const int len = a.row_len[row];
  const int npages = (len + kPage - 1) / kPage;
  const int per = (npages + a.splits - 1) / a.splits;
  const int pb = split * per;
  const int npg = max(0, min(npages, pb + per) - pb);  // pages of this CTA
  const int* bt = a.block_tables + (size_t)seq * a.max_blocks;

  if (warp == NW) {
    // ---------------------------------------------------------------- copy warp
    const TC* cache = static_cast<const TC*>(a.cache);
    constexpr int PIECES = kPage * kRow / 8;  // 16-byte pieces per page (1152: 36 per lane)
    int pg = 0;                              // block-table entries fetched 32 at a time
    for (int i = 0; i < npg; ++i) {
      const int s = i % kMlaRing;
      if ((i & 31) == 0) pg = i + lane < npg ? bt[pb + i + lane] : 0;
      int phys = __shfl_sync(0xffffffffu, pg, i & 31);
      if (a.num_blocks > 0 && (phys < 0 || phys >= a.num_blocks)) {  // bad block-table entry
        if (lane == 0 && a.err) atomicExch(a.err, 0xA00);
        phys = 0;
      }
      bool ok = true;
      if (i >= kMlaRing) {
        if (lane == 0) ok = tc::mbar_wait(&empty[s], ((i / kMlaRing) - 1) & 1, err, 1);
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      if (!ok) break;
      const TC* src = cache + (size_t)phys * kPage * kRow;
      TC* dst = reinterpret_cast<TC*>(ring + s * R::PAGE);
      for (int pc = lane; pc < PIECES; pc += 32) {
        const int r = pc / (kRow / 8), c = (pc % (kRow / 8)) * 8;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst + r * kMlaLd + c)),
                     "l"(src + r * kRow + c));
      }
      asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[s])) : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");  // copies land before the CTA exits
  } else {
    // ---------------------------------------------------------------- compute warps
    const int g = lane >> 2, tig = lane & 3;
    uint32_t qf[KSW][4];
#pragma unroll
    for (int kk = 0; kk < KSW; ++kk) {
      const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = (warp * KSW + kk) * 16 + (lane >> 4) * 8;
      ldsm_x4(qf[kk], smem_u32(sQ + r * kMlaLd + c));
    }
    float o[NDW][4];
#pragma unroll
    for (int j = 0; j < NDW; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m0 = -1e30f, m1 = -1e30f, l0 = 0.f, l1 = 0.f;  // heads g and g + 8
    for (int i = 0; i < npg; ++i) {
      const int s = i % kMlaRing;
      bool ok = !*err && tc::mbar_wait(&full[s], (uint32_t)((i / kMlaRing) & 1), err, 2);
      ok = __all_sync(0xffffffffu, ok);
      const TC* page = reinterpret_cast<const TC*>(ring + s * R::PAGE);
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      if (ok) {
#pragma unroll
        for (int kk = 0; kk < KSW; ++kk) {
          uint32_t kf[4];
          const int r = (lane & 7) + (lane >> 4) * 8;
          const int c = (warp * KSW + kk) * 16 + ((lane >> 3) & 1) * 8;
          ldsm_x4(kf, smem_u32(page + r * kMlaLd + c));
          MmaT<TC>::mma(sc[0], qf[kk], kf);
          MmaT<TC>::mma(sc[1], qf[kk], kf + 2);
        }
      }
      float* xw = sx + ((i & 1) * NW + warp) * 256;  // this warp's partial, [head][token]
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        *reinterpret_cast<float2*>(xw + g * 16 + j * 8 + 2 * tig) = make_float2(sc[j][0], sc[j][1]);
        *reinterpret_cast<float2*>(xw + (g + 8) * 16 + j * 8 + 2 * tig) = make_float2(sc[j][2], sc[j][3]);
      }
      if (!ok && lane == 0) stop[i & 1] = 1;
      asm volatile("bar.sync 1, 128;" ::: "memory");  // the four compute warps
      if (stop[i & 1]) break;                         // read after the barrier: the same in every warp
      // full scores: the four partials added in warp order (identical in every warp)
      const float* x0 = sx + (i & 1) * NW * 256;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int off = (g + 8 * hh) * 16 + j * 8 + 2 * tig;
          float2 v = *reinterpret_cast<const float2*>(x0 + off);
#pragma unroll
          for (int w = 1; w < NW; ++w) {
            const float2 u = *reinterpret_cast<const float2*>(x0 + w * 256 + off);
            v.x += u.x;
            v.y += u.y;
          }
          sc[j][2 * hh] = v.x;
          sc[j][2 * hh + 1] = v.y;
        }
      // mask + online softmax of heads g (entries 0, 1) and g + 8 (entries 2, 3), log2 domain
      float mn0 = m0, mn1 = m1;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int tok = (pb + i) * kPage + j * 8 + 2 * tig + (e & 1);
          const float v = tok < len ? sc[j][e] * kLog2e : -INFINITY;
          sc[j][e] = v;
          if (e < 2) mn0 = fmaxf(mn0, v);
          else mn1 = fmaxf(mn1, v);
        }
      mn0 = fmaxf(mn0, __shfl_xor_sync(0xffffffffu, mn0, 1));
      mn0 = fmaxf(mn0, __shfl_xor_sync(0xffffffffu, mn0, 2));
      mn1 = fmaxf(mn1, __shfl_xor_sync(0xffffffffu, mn1, 1));
      mn1 = fmaxf(mn1, __shfl_xor_sync(0xffffffffu, mn1, 2));
      const float c0 = exp2f(m0 - mn0), c1 = exp2f(m1 - mn1);
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float p = exp2f(sc[j][e] - (e < 2 ? mn0 : mn1));
          sc[j][e] = p;
          if (e < 2) ps0 += p;
          else ps1 += p;
        }
      ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
      ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
      ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
      ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
      l0 = l0 * c0 + ps0;
      l1 = l1 * c1 + ps1;
      m0 = mn0;
      m1 = mn1;
#pragma unroll
      for (int j = 0; j < NDW; ++j) {
        o[j][0] *= c0;
        o[j][1] *= c0;
        o[j][2] *= c1;
        o[j][3] *= c1;
      }
      // O[:, this warp's 128 dims] += P C (16 tokens = one k-step); P straight from the S fragments
      uint32_t pf[4];
      pf[0] = MmaT<TC>::pack(sc[0][0], sc[0][1]);
      pf[1] = MmaT<TC>::pack(sc[0][2], sc[0][3]);
      pf[2] = MmaT<TC>::pack(sc[1][0], sc[1][1]);
      pf[3] = MmaT<TC>::pack(sc[1][2], sc[1][3]);
#pragma unroll
      for (int jd = 0; jd < NDW; jd += 2) {
        uint32_t vf[4];
        const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = warp * (kLat / NW) + jd * 8 + (lane >> 4) * 8;
        ldsm_x4_t(vf, smem_u32(page + r * kMlaLd + c));
        MmaT<TC>::mma(o[jd], pf, vf);
        MmaT<TC>::mma(o[jd + 1], pf, vf + 2);
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[s]);
    }
    // unnormalised split partial: this warp's 128 dims of heads g and g + 8; (m, l) in natural log
    const size_t p0 = ((size_t)row * a.splits + split) * kMlaHeads;
#pragma unroll
    for (int jd = 0; jd < NDW; ++jd) {
      const int d = warp * (kLat / NW) + jd * 8 + 2 * tig;
      *reinterpret_cast<float2*>(a.part_acc + (p0 + g) * kLat + d) = make_float2(o[jd][0], o[jd][1]);
      *reinterpret_cast<float2*>(a.part_acc + (p0 + g + 8) * kLat + d) = make_float2(o[jd][2], o[jd][3]);
    }
    if (warp == 0 && tig == 0) {
      a.part_ml[p0 + g] = make_float2(m0 * kLn2, l0);
      a.part_ml[p0 + g + 8] = make_float2(m1 * kLn2, l1);
    }
  }
  __syncthreads();  // every warp is past its waits (no early return above)
  if (threadIdx.x == 0 && err_s && a.err) atomicExch(a.err, err_s);  // a wait that ran out
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

template <typename TC>
static cudaError_t launch_mla_mma(const MlaAttnArgs& a, cudaStream_t st) {
  auto kern = mla_attn_mma_kernel<TC>;
  constexpr int smem = MlaRing<TC>::BYTES;
  static const cudaError_t attr = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (attr != cudaSuccess) return attr;
  return launch_pdl(kern, dim3(a.splits, a.rows), dim3(kMlaThreads), (size_t)smem, st, a);
}

int mla_attention(const MlaAttnArgs& a, int cache_is_bf16, cudaStream_t st, int impl) {
  if (a.H != kMlaHeads) return -1;
  if (a.splits < 1 || a.splits > 64) return -2;
  if (a.rows <= 0) return 0;
  if (impl == 1) {
    cudaError_t e = cache_is_bf16 ? launch_mla_mma<__nv_bfloat16>(a, st) : launch_mla_mma<__half>(a, st);
    if (e == cudaSuccess) e = launch_pdl(mla_merge_kernel, dim3(kMlaHeads, a.rows), dim3(256), 0, st, a);
    return e == cudaSuccess ? 0 : -20;
  }
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
