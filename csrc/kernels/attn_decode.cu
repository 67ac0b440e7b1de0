// K8: paged flash-decode attention (one new query token per sequence), GQA-packed, split-KV.
//
// The reference has no attention kernel at all: FlashAttention::forward* returns Unsupported
// (backend/src/cuda_flash_attn.rs:165-359) and the CPU path loops over heads and query rows
// (models/src/transformer.rs:301-374).
//
// Grid (splits, Hkv, B), 4 compute warps + 1 copy warp per CTA.  All G = H/Hkv query heads of a KV
// head share one CTA, so every K/V page (16 tokens x D) is read from HBM once per step.  The copy
// warp streams the CTA's pages (cp.async, 16-byte pieces into rows padded for conflict-free
// ldmatrix; an fp8 cache is widened to fp16 on the way) into a 6-slot shared-memory ring ahead of
// the compute warps, which signal per slot through mbarriers.  Compute warp w takes pages w, w+4,
// ...: S = Q K^T for the G query heads (MMA rows, padded to 16) x 16 tokens on the tensor cores
// (mma.m16n8k16, fp32 accumulate, 2 x D/16 MMAs), online softmax in the log2 domain on the
// accumulator fragments, O += P V (D/8 MMAs) with P taken straight from the S fragments.  The CTA
// merges its 4 warps and writes an unnormalized partial per split.
// The splits are then merged (normalized, written as bf16/fp16 and as the int8 q8 activation of
// the output projection) by the last split CTA of each (sequence, KV head) to arrive -- a counter
// per (b, kv head) finds it, and it resets the counter -- or, without counters, by a second kernel.
#include "common.cuh"
#include "pdl.cuh"
#include "launch.h"
#include "tc_common.cuh"
#include "mma_sync.cuh"

#include <type_traits>

namespace barq {

constexpr int kBS = 16;  // tokens per KV page

constexpr int kAttnRing = 6;       // shared-memory page slots per CTA (3 CTAs per SM fit)
constexpr int kAttnRingDeep = 12;  // opt-in (BARQ_ATTN_RING=12): twice the bytes in flight per CTA, 2 CTAs per SM
constexpr int kAttnThreads = 160;  // 4 compute warps + 1 copy warp

// Ring layout: per slot one K page and one V page of 16 tokens x D operands (fp16 / bf16; an fp8
// cache is widened to fp16 by the copy warp), rows padded to D + 8 elements so that ldmatrix reads
// are bank-conflict free.
template <typename TM, int D, int RING = kAttnRing>
struct AttnRing {
  static constexpr int LD = D + 8;
  static constexpr int PAGE = kBS * LD * (int)sizeof(TM);
  static constexpr int SLOT = 2 * PAGE;
  static constexpr int QBYTES = 16 * LD * (int)sizeof(TM);  // the (padded) query heads, after the ring
  static constexpr int BYTES = RING * SLOT + QBYTES;
};

// TC: cache element type; TM: tensor-core operand type (TC for fp16 / bf16, fp16 for fp8).
template <typename TC, typename TM, int D, int G, int RING>
__global__ void __launch_bounds__(kAttnThreads) decode_attn_kernel(DecodeAttnArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int NW = 4;
  constexpr int KS = D / 16;  // k-steps of QK^T
  constexpr int ND = D / 8;   // O n-blocks
  using R = AttnRing<TM, D, RING>;
  static_assert(4 * G * D * (int)sizeof(float) <= RING * R::SLOT, "the warp merge aliases the ring");
  constexpr int LD = R::LD;
  static_assert(G <= 8, "query heads of a KV head fit the first 8 MMA rows");
  const int split = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float sl2 = a.scale * 1.4426950408889634f;

  extern __shared__ __align__(128) uint8_t ring[];
  TM* sQ = reinterpret_cast<TM*>(ring + RING * R::SLOT);
  __shared__ __align__(8) uint64_t full[RING], empty[RING];
  __shared__ float m_s[NW][G], l_s[NW][G];
  __shared__ int err_s;

  if (threadIdx.x == 0) {
    err_s = 0;
    for (int i = 0; i < RING; ++i) {
      tc::mbar_init(&full[i], 32);  // one arrival per copy-warp lane
      tc::mbar_init(&empty[i], 1);
    }
    tc::fence_mbar_init();
  }
  for (int i = threadIdx.x; i < 16 * D; i += blockDim.x) {  // query heads as MMA rows 0..G-1
    const int r = i / D, d = i % D;
    sQ[r * LD + d] = from_f<TM>(r < G ? __bfloat162float(a.q[((size_t)b * a.H + kvh * G + r) * D + d]) : 0.f);
  }
  __syncthreads();
  volatile int* err = &err_s;

  const int seq_len = a.seq_lens[b];
  const int first_tok = a.window > 0 ? max(0, seq_len - a.window) : 0;
  const int blk0 = first_tok / kBS;
  const int nblk = (seq_len + kBS - 1) / kBS - blk0;
  const int per = (nblk + a.splits - 1) / a.splits;
  const int sb = blk0 + split * per;
  const int npg = max(0, min(blk0 + nblk, sb + per) - sb);  // pages of this CTA
  const int* bt = a.block_tables + (size_t)b * a.max_blocks;

  const int g = lane >> 2, tig = lane & 3;
  float o[ND][4];
#pragma unroll
  for (int j = 0; j < ND; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mrow = -1e30f, lrow = 0.f;  // row g (rows g + 8 are padding)

  if (warp == NW) {
    // ---------------------------------------------------------------- copy warp
    // Every lane copies 1/32 of each page pair (16-byte pieces into the padded rows) and arrives on
    // the slot's barrier once its copies have landed.
    const TC* kc = static_cast<const TC*>(a.kcache);
    const TC* vc = static_cast<const TC*>(a.vcache);
    constexpr int PIECES = kBS * D / 8;  // 8-element pieces per page
    int pg = 0;  // physical page of entry (i & ~31) + lane: block-table entries fetched 32 at a time
    for (int i = 0; i < npg; ++i) {
      const int s = i % RING;
      if ((i & 31) == 0) pg = i + lane < npg ? bt[sb + i + lane] : 0;
      int phys = __shfl_sync(0xffffffffu, pg, i & 31);
      if (a.num_blocks > 0 && (phys < 0 || phys >= a.num_blocks)) {  // bad block-table entry
        if (lane == 0 && a.err) atomicExch(a.err, 0xA00);
        phys = 0;
      }
      bool ok = true;
      if (i >= RING) {
        if (lane == 0) ok = tc::mbar_wait(&empty[s], ((i / RING) - 1) & 1, err, 1);
        ok = __shfl_sync(0xffffffffu, ok, 0);
      }
      if (!ok) break;
      const size_t page = ((size_t)phys * a.Hkv + kvh) * kBS * D;
      TM* dk = reinterpret_cast<TM*>(ring + s * R::SLOT);
      TM* dv = reinterpret_cast<TM*>(ring + s * R::SLOT + R::PAGE);
      for (int pc = lane; pc < PIECES; pc += 32) {
        const int r = pc / (D / 8), c = (pc % (D / 8)) * 8;
        if constexpr (std::is_same<TC, TM>::value) {
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dk + r * LD + c)),
                       "l"(kc + page + r * D + c));
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dv + r * LD + c)),
                       "l"(vc + page + r * D + c));
        } else {  // fp8 cache: 8 elements -> 8 fp16 operands
          const uint2 rk = __ldg(reinterpret_cast<const uint2*>(kc + page + r * D + c));
          const uint2 rv = __ldg(reinterpret_cast<const uint2*>(vc + page + r * D + c));
          const TC* ek = reinterpret_cast<const TC*>(&rk);
          const TC* ev = reinterpret_cast<const TC*>(&rv);
          const size_t srow = ((size_t)phys * a.Hkv + kvh) * kBS + r;  // per-row scales (or unscaled)
          const float ks = a.kscale ? a.kscale[srow] : 1.f, vs = a.vscale ? a.vscale[srow] : 1.f;
          TM tk[8], tv[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            tk[j] = from_f<TM>(to_f(ek[j]) * ks);
            tv[j] = from_f<TM>(to_f(ev[j]) * vs);
          }
          *reinterpret_cast<int4*>(dk + r * LD + c) = *reinterpret_cast<int4*>(tk);
          *reinterpret_cast<int4*>(dv + r * LD + c) = *reinterpret_cast<int4*>(tv);
        }
      }
      if constexpr (std::is_same<TC, TM>::value)
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(&full[s])) : "memory");
      else
        tc::mbar_arrive(&full[s]);
    }
    // copies in flight land before the ring is reused or the CTA exits
    asm volatile("cp.async.wait_all;" ::: "memory");
  } else {
    // ---------------------------------------------------------------- compute warps (mma.m16n8k16)
    uint32_t qf[KS][4];
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
      const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
      const int c = kk * 16 + (lane >> 4) * 8;
      ldsm_x4(qf[kk], smem_u32(sQ + r * LD + c));
    }
    for (int i = warp; i < npg; i += NW) {
      const int s = i % RING;
      if (*err || !tc::mbar_wait(&full[s], (uint32_t)((i / RING) & 1), err, 2)) break;
      const TM* k_s = reinterpret_cast<const TM*>(ring + s * R::SLOT);
      const TM* v_s = reinterpret_cast<const TM*>(ring + s * R::SLOT + R::PAGE);
      // S = Q K^T: 16 (head) rows x 16 tokens
      float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
      for (int kk = 0; kk < KS; ++kk) {
        uint32_t kf[4];
        const int r = (lane & 7) + (lane >> 4) * 8;
        const int c = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(kf, smem_u32(k_s + r * LD + c));
        MmaT<TM>::mma(sc[0], qf[kk], kf);
        MmaT<TM>::mma(sc[1], qf[kk], kf + 2);
      }
      // mask + online softmax of row g (log2 domain)
      float mnew = mrow;
#pragma unroll
      for (int j = 0; j < 2; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int kpos = (sb + i) * kBS + j * 8 + 2 * tig + e;
          const bool ok = kpos < seq_len && kpos >= first_tok;
          const float v = ok ? sc[j][e] * sl2 : -INFINITY;
          sc[j][e] = v;
          mnew = fmaxf(mnew, v);
        }
      mnew = fmaxf(mnew, __shfl_xor_sync(0xffffffffu, mnew, 1));
      mnew = fmaxf(mnew, __shfl_xor_sync(0xffffffffu, mnew, 2));
      const float corr = exp2f(mrow - mnew);
      float psum = 0.f;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const float p = exp2f(sc[j][e] - mnew);
          sc[j][e] = p;
          psum += p;
        }
        sc[j][2] = sc[j][3] = 0.f;  // padding rows g + 8
      }
      psum += __shfl_xor_sync(0xffffffffu, psum, 1);
      psum += __shfl_xor_sync(0xffffffffu, psum, 2);
      lrow = lrow * corr + psum;
      mrow = mnew;
#pragma unroll
      for (int j = 0; j < ND; ++j) {
        o[j][0] *= corr;
        o[j][1] *= corr;
      }
      // O += P V (16 tokens = one k-step)
      uint32_t pf[4];
      pf[0] = MmaT<TM>::pack(sc[0][0], sc[0][1]);
      pf[1] = MmaT<TM>::pack(sc[0][2], sc[0][3]);
      pf[2] = MmaT<TM>::pack(sc[1][0], sc[1][1]);
      pf[3] = MmaT<TM>::pack(sc[1][2], sc[1][3]);
#pragma unroll
      for (int jd = 0; jd < ND; jd += 2) {
        uint32_t vf[4];
        const int r = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = jd * 8 + (lane >> 4) * 8;
        ldsm_x4_t(vf, smem_u32(v_s + r * LD + c));
        MmaT<TM>::mma(o[jd], pf, vf);
        MmaT<TM>::mma(o[jd + 1], pf, vf + 2);
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&empty[s]);
    }
  }
  __syncthreads();  // the ring is free: every page was consumed and the copies drained
  float(*acc_s)[G][D] = reinterpret_cast<float(*)[G][D]>(ring);  // [NW][G][D], aliases the ring
  // merge the 4 compute warps of this CTA: rows g < G of each warp's O, m and l
  if (warp < NW && g < G) {
    if (tig == 0) {
      m_s[warp][g] = mrow;
      l_s[warp][g] = lrow;
    }
#pragma unroll
    for (int j = 0; j < ND; ++j) {
      acc_s[warp][g][j * 8 + 2 * tig] = o[j][0];
      acc_s[warp][g][j * 8 + 2 * tig + 1] = o[j][1];
    }
  }
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

template <typename TC, int D, int G, int RING>
static cudaError_t launch_attn_ring(const DecodeAttnArgs& a, dim3 grid, cudaStream_t st) {
  using TM = typename std::conditional<std::is_same<TC, __nv_fp8_e4m3>::value, __half, TC>::type;
  auto kern = decode_attn_kernel<TC, TM, D, G, RING>;
  constexpr int smem = AttnRing<TM, D, RING>::BYTES;
  static const cudaError_t attr = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (attr != cudaSuccess) return attr;
  return launch_pdl(kern, grid, dim3(kAttnThreads), (size_t)smem, st, a);
}

// ring depth: 6 slots (default), or 12 with BARQ_ATTN_RING=12 (not yet measured on a GPU)
static int attn_ring_depth() {
  static const int depth = [] {
    const char* e = getenv("BARQ_ATTN_RING");
    return e && atoi(e) == kAttnRingDeep ? kAttnRingDeep : kAttnRing;
  }();
  return depth;
}

template <typename TC, int D, int G>
static cudaError_t launch_attn(const DecodeAttnArgs& a, dim3 grid, cudaStream_t st) {
  return attn_ring_depth() == kAttnRingDeep ? launch_attn_ring<TC, D, G, kAttnRingDeep>(a, grid, st)
                                            : launch_attn_ring<TC, D, G, kAttnRing>(a, grid, st);
}

template <typename TC, int D>
static int launch_g(const DecodeAttnArgs& a, cudaStream_t st) {
  const int G = a.H / a.Hkv;
  dim3 grid(a.splits, a.Hkv, a.B);
  cudaError_t e;
  switch (G) {
    case 1: e = launch_attn<TC, D, 1>(a, grid, st); break;
    case 2: e = launch_attn<TC, D, 2>(a, grid, st); break;
    case 4: e = launch_attn<TC, D, 4>(a, grid, st); break;
    case 8: e = launch_attn<TC, D, 8>(a, grid, st); break;
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
