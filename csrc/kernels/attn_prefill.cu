// K9: causal varlen prefill attention over the paged KV cache (chunked prefill aware), GQA, SWA.
//
// FlashAttention-2 structure: a CTA owns 64 query rows of one head (16 per warp); K/V tiles of 64
// tokens (4 pages) are staged in shared memory with cp.async (double-buffered); S = QK^T and
// O += PV run on the tensor cores (mma.m16n8k16, fp32 accumulate) with P kept in registers;
// the softmax is online in the log2 domain.  Query row i of a sequence sits at absolute position
// ctx_len - n_new + i, so the same kernel serves first prefill and later prefill chunks.
//
// The reference's only attention is a per-row CPU loop (models/src/transformer.rs:301-374) and a
// CPU FA-2 (advanced/src/flash_attention.rs:169-271); its CUDA flash attention returns
// Unsupported (backend/src/cuda_flash_attn.rs:165-359).
#include <type_traits>

#include "common.cuh"
#include "pdl.cuh"
#include "launch.h"
#include "mma_sync.cuh"

namespace barq {

BARQ_DEV void cp_async16(void* dst, const void* src, bool pred) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(pred ? 16 : 0));
}
BARQ_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N> BARQ_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N)); }

// TC: KV cache element type; TM: tensor-core operand type (TC itself for fp16/bf16; fp16 for an
// fp8 cache, whose pages are converted while being staged in shared memory).
template <typename TC, typename TM, int D>
__global__ void __launch_bounds__(128) prefill_attn_kernel(PrefillAttnArgs a) {
  pdl_wait();
  pdl_trigger();
  constexpr int BQ = 64, BK = 64, LD = D + 8;  // padded rows (16 B) avoid ldmatrix bank conflicts
  constexpr int NB = BK / 8;                   // S n-blocks per warp
  constexpr int KS = D / 16;                   // k-steps of QK^T
  constexpr int ND = D / 8;                    // O n-blocks
  extern __shared__ __align__(16) unsigned char smem_raw[];
  TM* sQ = reinterpret_cast<TM*>(smem_raw);
  TM* sK = sQ + BQ * LD;           // [2][BK][LD]
  TM* sV = sK + 2 * BK * LD;       // [2][BK][LD]

  const int s = blockIdx.z, h = blockIdx.y, qt = blockIdx.x;
  const int q_begin = a.q_start[s], n_new = a.q_start[s + 1] - q_begin;
  const int q0 = qt * BQ;
  if (q0 >= n_new) return;
  const int ctx = a.ctx_lens[s];
  const int base_pos = ctx - n_new;
  const int G = a.H / a.Hkv, kvh = h / G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  const float sl2 = a.scale * 1.4426950408889634f;

  // ---- Q tile -> smem (converted to the cache element type)
  for (int i = tid; i < BQ * D / 8; i += 128) {
    int r = i / (D / 8), c = (i % (D / 8)) * 8;
    int qi = q0 + r;
    TM tmp[8];
    if (qi < n_new) {
      const __nv_bfloat16* src = a.q + ((size_t)(q_begin + qi) * a.H + h) * D + c;
      int4 raw = *reinterpret_cast<const int4*>(src);
      const __nv_bfloat16* hv = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) tmp[j] = from_f<TM>(__bfloat162float(hv[j]));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) tmp[j] = from_f<TM>(0.f);
    }
    *reinterpret_cast<int4*>(sQ + r * LD + c) = *reinterpret_cast<int4*>(tmp);
  }

  const int q_last = min(q0 + BQ, n_new) - 1;
  const int kv_end = base_pos + q_last + 1;  // exclusive, causal
  int kv_begin = 0;
  if (a.window > 0) kv_begin = max(0, base_pos + q0 - a.window + 1);
  const int t_begin = kv_begin / BK, t_end = (kv_end + BK - 1) / BK;
  const int* bt = a.block_tables + (size_t)s * a.max_blocks;
  const TC* kc = reinterpret_cast<const TC*>(a.kcache);
  const TC* vc = reinterpret_cast<const TC*>(a.vcache);

  auto load_kv = [&](int tile, int buf) {
    TM* dk = sK + buf * BK * LD;
    TM* dv = sV + buf * BK * LD;
    for (int i = tid; i < BK * D / 8; i += 128) {
      int r = i / (D / 8), c = (i % (D / 8)) * 8;
      int pos = tile * BK + r;
      bool ok = pos < kv_end;
      int phys = ok ? bt[pos >> 4] : 0;
      size_t off = (((size_t)phys * a.Hkv + kvh) * 16 + (pos & 15)) * D + c;
      if constexpr (std::is_same<TC, TM>::value) {
        cp_async16(dk + r * LD + c, kc + off, ok);
        cp_async16(dv + r * LD + c, vc + off, ok);
      } else {  // fp8 cache: 8 elements (8 bytes) -> 8 operands (16 bytes)
        TM tk[8], tv[8];
        if (ok) {
          const uint2 rk = __ldg(reinterpret_cast<const uint2*>(kc + off));
          const uint2 rv = __ldg(reinterpret_cast<const uint2*>(vc + off));
          const TC* ek = reinterpret_cast<const TC*>(&rk);
          const TC* ev = reinterpret_cast<const TC*>(&rv);
          const size_t srow = ((size_t)phys * a.Hkv + kvh) * 16 + (pos & 15);  // per-row scales
          const float ks = a.kscale ? a.kscale[srow] : 1.f, vs = a.vscale ? a.vscale[srow] : 1.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            tk[j] = from_f<TM>(to_f(ek[j]) * ks);
            tv[j] = from_f<TM>(to_f(ev[j]) * vs);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) tk[j] = tv[j] = from_f<TM>(0.f);
        }
        *reinterpret_cast<int4*>(dk + r * LD + c) = *reinterpret_cast<int4*>(tk);
        *reinterpret_cast<int4*>(dv + r * LD + c) = *reinterpret_cast<int4*>(tv);
      }
    }
    cp_async_commit();
  };

  if (t_begin < t_end) load_kv(t_begin, 0);
  __syncthreads();

  // Q fragments (16 rows of this warp) for all k-steps
  uint32_t qf[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    int c = kk * 16 + (lane >> 4) * 8;
    ldsm_x4(qf[kk], smem_u32(sQ + r * LD + c));
  }

  float o[ND][4];
#pragma unroll
  for (int j = 0; j < ND; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float mrow[2] = {-1e30f, -1e30f}, lrow[2] = {0.f, 0.f};
  const int g = lane >> 2, tig = lane & 3;
  const int qpos0 = base_pos + q0 + warp * 16 + g;  // absolute position of row g (row g+8: +8)

  for (int t = t_begin; t < t_end; ++t) {
    const int buf = (t - t_begin) & 1;
    if (t + 1 < t_end) {
      load_kv(t + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const TM* k_s = sK + buf * BK * LD;
    const TM* v_s = sV + buf * BK * LD;
    float sc[NB][4];
#pragma unroll
    for (int j = 0; j < NB; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
      for (int jp = 0; jp < NB; jp += 2) {
        uint32_t kf[4];
        int r = jp * 8 + (lane & 7) + (lane >> 4) * 8;
        int c = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(kf, smem_u32(k_s + r * LD + c));
        MmaT<TM>::mma(sc[jp], qf[kk], kf);
        MmaT<TM>::mma(sc[jp + 1], qf[kk], kf + 2);
      }
    }
    // mask + online softmax
    float mnew[2] = {mrow[0], mrow[1]};
#pragma unroll
    for (int j = 0; j < NB; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        int kpos = t * BK + j * 8 + 2 * tig + (e & 1);
        int qpos = qpos0 + (e >> 1) * 8;
        bool ok = kpos <= qpos && kpos < kv_end && (a.window <= 0 || kpos > qpos - a.window);
        float v = ok ? sc[j][e] * sl2 : -INFINITY;
        sc[j][e] = v;
        mnew[e >> 1] = fmaxf(mnew[e >> 1], v);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 1));
      mnew[r] = fmaxf(mnew[r], __shfl_xor_sync(0xffffffffu, mnew[r], 2));
    }
    float corr[2], psum[2] = {0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 2; ++r) corr[r] = exp2f(mrow[r] - mnew[r]);
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float p = exp2f(sc[j][e] - mnew[e >> 1]);
        sc[j][e] = p;
        psum[e >> 1] += p;
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 1);
      psum[r] += __shfl_xor_sync(0xffffffffu, psum[r], 2);
      lrow[r] = lrow[r] * corr[r] + psum[r];
      mrow[r] = mnew[r];
    }
#pragma unroll
    for (int j = 0; j < ND; ++j) {
      o[j][0] *= corr[0];
      o[j][1] *= corr[0];
      o[j][2] *= corr[1];
      o[j][3] *= corr[1];
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BK / 16; ++kk) {
      uint32_t pf[4];
      pf[0] = MmaT<TM>::pack(sc[2 * kk][0], sc[2 * kk][1]);
      pf[1] = MmaT<TM>::pack(sc[2 * kk][2], sc[2 * kk][3]);
      pf[2] = MmaT<TM>::pack(sc[2 * kk + 1][0], sc[2 * kk + 1][1]);
      pf[3] = MmaT<TM>::pack(sc[2 * kk + 1][2], sc[2 * kk + 1][3]);
#pragma unroll
      for (int jd = 0; jd < ND; jd += 2) {
        uint32_t vf[4];
        int r = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        int c = jd * 8 + (lane >> 4) * 8;
        ldsm_x4_t(vf, smem_u32(v_s + r * LD + c));
        MmaT<TM>::mma(o[jd], pf, vf);
        MmaT<TM>::mma(o[jd + 1], pf, vf + 2);
      }
    }
    __syncthreads();
  }
  // write out
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    int qi = q0 + warp * 16 + g + r * 8;
    if (qi >= n_new) continue;
    float inv = lrow[r] > 0.f ? 1.f / lrow[r] : 0.f;
    const size_t base = ((size_t)(q_begin + qi) * a.H + h) * D;
#pragma unroll
    for (int j = 0; j < ND; ++j) {
      const float v0 = o[j][2 * r] * inv, v1 = o[j][2 * r + 1] * inv;
      if (a.out_f16) {
        *reinterpret_cast<__half2*>(reinterpret_cast<__half*>(a.out) + base + j * 8 + 2 * tig) = __floats2half2_rn(v0, v1);
      } else {
        *reinterpret_cast<__nv_bfloat162*>(reinterpret_cast<__nv_bfloat16*>(a.out) + base + j * 8 + 2 * tig) =
            __floats2bfloat162_rn(v0, v1);
      }
    }
  }
}

template <typename TC, typename TM, int D>
static int launch_prefill(const PrefillAttnArgs& a, cudaStream_t st) {
  constexpr int LD = D + 8;
  size_t smem = (size_t)(64 * LD + 4 * 64 * LD) * sizeof(TM);
  if (cudaFuncSetAttribute(prefill_attn_kernel<TC, TM, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
      cudaSuccess)
    return -12;
  dim3 grid((a.max_q + 63) / 64, a.H, a.S);
  return launch_pdl(prefill_attn_kernel<TC, TM, D>, grid, dim3(128), smem, st, a) == cudaSuccess ? 0 : -20;
}

int prefill_attention(const PrefillAttnArgs& a, cudaStream_t st) {
  if (a.block_size != 16) return -1;
  if (a.S <= 0 || a.max_q <= 0) return 0;
  if (a.impl == 1) {
    const int rc = prefill_attention_tc(a, st);
    if (rc != -2) return rc;
  }
  if (a.D == 128)
    return a.cache_type == kCacheBF16  ? launch_prefill<__nv_bfloat16, __nv_bfloat16, 128>(a, st)
           : a.cache_type == kCacheFP8 ? launch_prefill<__nv_fp8_e4m3, __half, 128>(a, st)
                                       : launch_prefill<__half, __half, 128>(a, st);
  if (a.D == 64)
    return a.cache_type == kCacheBF16  ? launch_prefill<__nv_bfloat16, __nv_bfloat16, 64>(a, st)
           : a.cache_type == kCacheFP8 ? launch_prefill<__nv_fp8_e4m3, __half, 64>(a, st)
                                       : launch_prefill<__half, __half, 64>(a, st);
  return -4;
}

}  // namespace barq
