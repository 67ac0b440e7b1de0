// K9 on the 5th-generation tensor cores: causal varlen prefill attention over the paged KV cache
// with tcgen05.mma, TMEM accumulators and TMA-fed K/V tiles (fp16 / bf16 caches, D = 64 or 128).
//
// One CTA owns 128 query rows of one head (the 128 TMEM lanes) and walks the key tiles of 128
// tokens (8 pages) that its rows can see.  Roles, 6 warps:
//   warp 0      TMA producer: per tile, 8 pages x D/64 boxes {64, 16} of K and of V from the
//               cache viewed as a 2D tensor [blocks * Hkv * 16, D] (128-byte swizzle), 2 stages;
//   warp 1      MMA issuer (one thread) and TMEM owner:
//                 S_j = Q K_j^T    (SS: Q and K K-major in shared memory) into TMEM buffer j % 2,
//                 O  += P_j V_j    (TS: P from TMEM, V as an MN-major B operand) into TMEM O;
//               S_{j+1} is issued before P_j is ready, so the next scores overlap the softmax;
//   warps 2..5  softmax: thread r owns query row r (TMEM lane r).  It reads its S row, masks
//               (causal, sequence end, sliding window), keeps a running max m and sum l in the
//               log2 domain, writes P (packed two 16-bit values per column) over the S columns it
//               has read, and finally reads O, divides by l and stores the output row.
// TMEM (512 columns): S buffers at columns 0 and 128, O at column 256 (D columns).
//
// O is rescaled lazily: the running max used for the exponentials only moves when a row's new max
// exceeds it by more than 8 (a factor 256 in P), and the rescale of that row's O waits for the
// previous P V to finish (the softmax warps wait for every P V in turn, so nothing overwrites O
// while it is being rescaled).  Both l and O always refer to the same max, so the result is exact
// up to rounding whatever the threshold.
//
// Key positions beyond the last page of the sequence load the last page again (finite cache
// contents; their probabilities are exactly 0).  Every mbarrier wait is bounded; a timeout sets
// the error word and all roles unwind, with copies and MMAs in flight drained before TMEM is freed.
//
// The reference names flash_attn / flash_attn_causal / flash_attn_window
// (backend/src/cuda_flash_attn.rs:93-104) and returns Unsupported from all of them
// (backend/src/cuda_flash_attn.rs:165-359); its working attention is a CPU FA-2
// (advanced/src/flash_attention.rs:169-271).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "common.cuh"
#include "launch.h"
#include "pdl.cuh"
#include "tc_common.cuh"

namespace barq {
using namespace tc;

constexpr int kPtRows = 128;    // query rows per CTA (TMEM lanes)
constexpr int kPtKeys = 128;    // keys per tile (8 pages of 16)
constexpr int kPtThreads = 192; // warp 0 TMA, warp 1 MMA, warps 2..5 softmax
constexpr int kPtStages = 2;
constexpr int kPtOCol = 256;    // TMEM column of O
constexpr float kPtRescale = 8.f;  // lazy-rescale threshold (log2 units)

template <int D>
struct PtSmem {
  static constexpr int ATOMS = D / 64;           // 128-byte swizzle atoms along D
  static constexpr int ATOM = 128 * 128;         // 128 rows x 64 elements (16 KB)
  static constexpr int TILE = ATOMS * ATOM;      // Q, or one K / V tile
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = TILE;
  static constexpr int OFF_V = OFF_K + kPtStages * TILE;
  static constexpr int OFF_BAR = OFF_V + kPtStages * TILE;
  static constexpr int NBAR = 5 * kPtStages + 2;
  static constexpr int OFF_TMEM = OFF_BAR + NBAR * 8;
  static constexpr int BYTES = OFF_TMEM + 16 + 1024;  // + slack for the 1024-byte alignment
  // at least ~114 KB so that one CTA (which allocates all 512 TMEM columns) runs per SM
  static constexpr int LAUNCH_BYTES = BYTES > 116 * 1024 ? BYTES : 116 * 1024;
};
static_assert(PtSmem<128>::LAUNCH_BYTES <= 227 * 1024, "shared memory budget");

template <typename T> BARQ_DEV uint32_t pack2(float lo, float hi);
template <> BARQ_DEV uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> BARQ_DEV uint32_t pack2<__half>(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int D, bool F16>
__global__ void __launch_bounds__(kPtThreads, 1)
    prefill_attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                           PrefillAttnArgs a, int cache_blocks, int* gerr) {
  using L = PtSmem<D>;
  using TM = typename std::conditional<F16, __half, __nv_bfloat16>::type;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* k_full = bars;                       // [2] K tile landed (TMA bytes)
  uint64_t* v_full = bars + kPtStages;           // [2] V tile landed
  uint64_t* kv_empty = bars + 2 * kPtStages;     // [2] P V of the stage's tile done (stage reusable)
  uint64_t* s_full = bars + 3 * kPtStages;       // [2] S buffer written
  uint64_t* p_full = bars + 4 * kPtStages;       // [2] P written by the 4 softmax warps
  uint64_t* o_done = bars + 5 * kPtStages;       // P V finished (one phase per tile)
  uint64_t* drain = o_done + 1;                  // issuer's final drain of its MMAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_TMEM);
  __shared__ int err_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = blockIdx.z, h = blockIdx.y;
  const int qt = gridDim.x - 1 - blockIdx.x;  // the longest (last) query tiles start first
  pdl_trigger();
  pdl_wait();  // q, the cache pages and the tables come from earlier kernels
  const int q_begin = a.q_start[s], n_new = a.q_start[s + 1] - q_begin;
  const int q0 = qt * kPtRows;
  if (q0 >= n_new) return;  // uniform over the CTA: before any barrier or TMEM allocation
  const int ctx = a.ctx_lens[s], base_pos = ctx - n_new;
  const int G = a.H / a.Hkv, kvh = h / G;
  const int q_last = min(q0 + kPtRows, n_new) - 1;
  const int kv_end = base_pos + q_last + 1;  // exclusive (causal)
  const int kv_begin = a.window > 0 ? max(0, base_pos + q0 - a.window + 1) : 0;
  const int t_begin = kv_begin / kPtKeys, t_end = (kv_end + kPtKeys - 1) / kPtKeys;
  const int nt = t_end - t_begin;  // >= 1: every row sees at least its own position
  const float sl2 = a.scale * 1.4426950408889634f;

  if (threadIdx.x == 0) {
    err_s = 0;
    for (int i = 0; i < kPtStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
    }
    mbar_init(o_done, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);

  // ---- Q tile -> shared memory (every thread), K-major 128-byte swizzle: 16-byte chunk c of row r
  // within a 64-element atom sits at chunk position c ^ (r % 8)
  for (int i = threadIdx.x; i < kPtRows * (D / 8); i += kPtThreads) {
    const int r = i / (D / 8), c = i % (D / 8);
    const int qi = q0 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (qi < n_new) {
      v = *reinterpret_cast<const uint4*>(a.q + ((size_t)(q_begin + qi) * a.H + h) * D + c * 8);
      if constexpr (F16) {
        const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
        uint4 w;
        uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
        for (int j = 0; j < 4; ++j) wp[j] = pack2<__half>(__bfloat162float(e[2 * j]), __bfloat162float(e[2 * j + 1]));
        v = w;
      }
    }
    *reinterpret_cast<uint4*>(smem + L::OFF_Q + (c >> 3) * L::ATOM + r * 128 + (((c & 7) ^ (r & 7)) << 4)) = v;
  }
  fence_proxy_async();  // generic-proxy writes of Q -> visible to the tensor cores
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  volatile int* err = &err_s;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
      const int* bt = a.block_tables + (size_t)s * a.max_blocks;
      const int pg_last = (kv_end - 1) >> 4;
      int issued = 0;
      for (int j = 0; j < nt && !*err; ++j) {
        const int st = j % kPtStages, ph = (j / kPtStages) & 1;
        if (j >= kPtStages && !mbar_wait(&kv_empty[st], ph ^ 1, err, 0x20)) break;
        const int t = t_begin + j;
        uint8_t* kd = smem + L::OFF_K + st * L::TILE;
        uint8_t* vd = smem + L::OFF_V + st * L::TILE;
        mbar_expect_tx(&k_full[st], L::TILE);
        mbar_expect_tx(&v_full[st], L::TILE);
        for (int p = 0; p < kPtKeys / 16; ++p) {
          const int pg = min(t * (kPtKeys / 16) + p, pg_last);
          int phys = bt[pg];
          if (phys < 0 || phys >= cache_blocks) {  // bad block-table entry: report, read block 0
            if (gerr) atomicExch(gerr, 0xA00);  // as decode attention
            phys = 0;
          }
          const int y = (phys * a.Hkv + kvh) * 16;
#pragma unroll
          for (int at = 0; at < L::ATOMS; ++at) {
            tma_load_2d(kd + at * L::ATOM + p * 2048, &kmap, at * 64, y, &k_full[st]);
            tma_load_2d(vd + at * L::ATOM + p * 2048, &vmap, at * 64, y, &v_full[st]);
          }
        }
        ++issued;
      }
      // copies still in flight land before the CTA can exit
      for (int j = max(0, issued - kPtStages); j < issued; ++j) {
        mbar_wait_bounded(&k_full[j % kPtStages], (j / kPtStages) & 1);
        mbar_wait_bounded(&v_full[j % kPtStages], (j / kPtStages) & 1);
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = F16 ? idesc_f16(128, kPtKeys) : idesc_bf16(128, kPtKeys);
      constexpr uint32_t id_o = (F16 ? idesc_f16(128, D) : idesc_bf16(128, D)) | kIdescBMajorMN;
      const uint32_t q_s = smem_addr(smem + L::OFF_Q);
      auto issue_s = [&](int j) -> bool {
        const int st = j % kPtStages;
        if (!mbar_wait(&k_full[st], (j / kPtStages) & 1, err, 0x21)) return false;
        tc_fence_after();
        const uint32_t k_s = smem_addr(smem + L::OFF_K + st * L::TILE);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const int at = ks >> 2, kk = ks & 3;  // atom along D, 16-element step inside it (32 bytes)
          mma_bf16(tmem + (uint32_t)(st * kPtKeys), umma_desc_sw128(q_s + at * L::ATOM + 32 * kk),
                   umma_desc_sw128(k_s + at * L::ATOM + 32 * kk), id_s, ks > 0);
        }
        mma_commit(&s_full[st]);
        return true;
      };
      bool ok = issue_s(0);
      for (int j = 0; ok && j < nt; ++j) {
        if (j + 1 < nt && !(ok = issue_s(j + 1))) break;
        const int st = j % kPtStages, ph = (j / kPtStages) & 1;
        if (!mbar_wait(&p_full[st], ph, err, 0x22) || !mbar_wait(&v_full[st], ph, err, 0x23)) break;
        tc_fence_after();
        const uint32_t v_s = smem_addr(smem + L::OFF_V + st * L::TILE);
        // O += P V: A = P (TMEM, 16 keys = 8 columns per step), B = V rows of 16 keys (2048 bytes)
#pragma unroll
        for (int kk = 0; kk < kPtKeys / 16; ++kk)
          mma_f16_ts(tmem + (uint32_t)kPtOCol, tmem + (uint32_t)(st * kPtKeys + kk * 8),
                     umma_desc_sw128_mn(v_s + kk * 2048, (uint32_t)L::ATOM), id_o, (j > 0) | (kk > 0));
        mma_commit(o_done);
        mma_commit(&kv_empty[st]);
      }
      mma_commit(drain);  // arrives once every MMA issued above has completed
      mbar_wait_bounded(drain, 0);
    }
  } else {
    // ---------------------------------------------------------------- softmax + epilogue (warps 2..5)
    const int quad = warp & 3, r = quad * 32 + lane;
    const uint32_t lanes = (uint32_t)(quad * 32) << 16;
    const int qi = q0 + r, qpos = base_pos + qi;
    const int hi = min(qpos + 1, kv_end);                             // keys [lo, hi) are visible
    const int lo = a.window > 0 ? max(0, qpos - a.window + 1) : 0;
    float m_use = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      const int st = j % kPtStages, ph = (j / kPtStages) & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[st], ph, err, 0x24));
      if (!ok) break;
      tc_fence_after();
      const uint32_t sa = tmem + lanes + (uint32_t)(st * kPtKeys);
      const int k0 = (t_begin + j) * kPtKeys;
      float mx = -INFINITY;
#pragma unroll
      for (int c0 = 0; c0 < kPtKeys; c0 += 32) {
        float v[32];
        tmem_ld32(sa + (uint32_t)c0, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int kp = k0 + c0 + i;
          if (kp >= lo && kp < hi) mx = fmaxf(mx, v[i]);
        }
      }
      mx *= sl2;
      // the previous P V must be complete before O is touched (and it is waited for once per tile,
      // which keeps this barrier's phases in step)
      if (j > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(o_done, (j - 1) & 1, err, 0x25));
        if (!ok) break;
        tc_fence_after();
      }
      const float m_new = fmaxf(m_use, mx);
      const bool resc = m_new > m_use + kPtRescale;  // false while the row has seen no visible key
      const float f = resc ? exp2f(m_use - m_new) : 1.f;  // 0 when m_use is still -inf
      if (j > 0 && __any_sync(0xffffffffu, resc)) {
#pragma unroll 1
        for (int c0 = 0; c0 < D; c0 += 32) {
          float o[32];
          tmem_ld32(tmem + lanes + (uint32_t)(kPtOCol + c0), o);
          uint4 w[8];
          uint32_t* wp = reinterpret_cast<uint32_t*>(w);
#pragma unroll
          for (int i = 0; i < 32; ++i) wp[i] = __float_as_uint(o[i] * f);
          tmem_st16(tmem + lanes + (uint32_t)(kPtOCol + c0), w);
          tmem_st16(tmem + lanes + (uint32_t)(kPtOCol + c0 + 16), w + 4);
        }
      }
      if (resc) {
        l *= f;
        m_use = m_new;
      }
      float sum = 0.f;
#pragma unroll
      for (int c0 = 0; c0 < kPtKeys; c0 += 32) {
        float v[32];
        tmem_ld32(sa + (uint32_t)c0, v);
        uint4 pk[4];
        uint32_t* pp = reinterpret_cast<uint32_t*>(pk);
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const int kp = k0 + c0 + i;
          const float p0 = (kp >= lo && kp < hi) ? exp2f(v[i] * sl2 - m_use) : 0.f;
          const float p1 = (kp + 1 >= lo && kp + 1 < hi) ? exp2f(v[i + 1] * sl2 - m_use) : 0.f;
          sum += p0 + p1;
          pp[i >> 1] = pack2<TM>(p0, p1);
        }
        // P of keys [c0, c0 + 32) -> columns [c0 / 2, c0 / 2 + 16) of this S buffer (already read)
        tmem_st16(sa + (uint32_t)(c0 >> 1), pk);
      }
      l += sum;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[st]);
    }
    if (ok) ok = __all_sync(0xffffffffu, mbar_wait(o_done, (nt - 1) & 1, err, 0x26));
    if (ok) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const bool store = qi < n_new;
      uint8_t* orow = reinterpret_cast<uint8_t*>(a.out) + (((size_t)(q_begin + (store ? qi : 0)) * a.H + h) * D) * 2;
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 32) {
        float o[32];
        tmem_ld32(tmem + lanes + (uint32_t)(kPtOCol + c0), o);
        if (!store) continue;
        uint4 w[4];
        uint32_t* wp = reinterpret_cast<uint32_t*>(w);
#pragma unroll
        for (int i = 0; i < 32; i += 2)
          wp[i >> 1] = a.out_f16 ? pack2<__half>(o[i] * inv, o[i + 1] * inv)
                                 : pack2<__nv_bfloat16>(o[i] * inv, o[i + 1] * inv);
#pragma unroll
        for (int i = 0; i < 4; ++i) reinterpret_cast<uint4*>(orow + c0 * 2)[i] = w[i];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && err_s && gerr) atomicExch(gerr, err_s);
}

// ------------------------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 pt_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Tensor map of one layer's K or V cache as a 2D [rows, D] tensor, box {64, 16} (half a page row
// block of one head), 128-byte swizzle.  Maps are cached by (address, rows, D, type): a layer's
// cache keeps its address for the engine's lifetime.
static int pt_cache_map(CUtensorMap* out, const void* base, long rows, int D, bool f16) {
  struct Key {
    const void* p;
    long rows;
    int d, f16;
    bool operator==(const Key& o) const { return p == o.p && rows == o.rows && d == o.d && f16 == o.f16; }
  };
  struct Hash {
    size_t operator()(const Key& k) const { return std::hash<const void*>()(k.p) ^ (size_t)k.rows * 31 ^ k.d; }
  };
  static std::mutex mu;
  static std::unordered_map<Key, CUtensorMap, Hash> maps;
  const Key key{base, rows, D, f16 ? 1 : 0};
  std::lock_guard<std::mutex> lk(mu);
  auto it = maps.find(key);
  if (it != maps.end()) {
    *out = it->second;
    return 0;
  }
  auto enc = pt_encode();
  if (!enc) return -10;
  cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)D * 2};
  cuuint32_t box[2] = {64, 16};
  cuuint32_t es[2] = {1, 1};
  CUtensorMap m;
  CUresult r = enc(&m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return -11;
  maps.emplace(key, m);
  *out = m;
  return 0;
}

template <int D, bool F16>
static int launch_prefill_tc(const PrefillAttnArgs& a, cudaStream_t st) {
  using L = PtSmem<D>;
  CUtensorMap km, vm;
  int rc = pt_cache_map(&km, a.kcache, a.cache_rows, D, F16);
  if (rc == 0) rc = pt_cache_map(&vm, a.vcache, a.cache_rows, D, F16);
  if (rc) return rc;
  auto kern = prefill_attn_tc_kernel<D, F16>;
  static const cudaError_t attr =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::LAUNCH_BYTES);
  if (attr != cudaSuccess) return -12;
  const int cache_blocks = (int)(a.cache_rows / ((long)a.Hkv * 16));
  dim3 grid((a.max_q + kPtRows - 1) / kPtRows, a.H, a.S);
  const cudaError_t e = launch_pdl(kern, grid, dim3(kPtThreads), (size_t)L::LAUNCH_BYTES, st, km, vm, a,
                                   cache_blocks, kernel_err_word());
  return e == cudaSuccess ? 0 : -13;
}

// 0 on success; -2 when the shape or cache type has no tcgen05 instantiation (fp8 caches and
// D other than 64 / 128 use the mma.sync kernel).
int prefill_attention_tc(const PrefillAttnArgs& a, cudaStream_t st) {
  if (a.block_size != 16 || a.cache_rows <= 0) return -1;
  if (a.S <= 0 || a.max_q <= 0) return 0;
  if (a.cache_type == kCacheFP8) return -2;
  const bool f16 = a.cache_type == kCacheF16;
  if (a.D == 128) return f16 ? launch_prefill_tc<128, true>(a, st) : launch_prefill_tc<128, false>(a, st);
  if (a.D == 64) return f16 ? launch_prefill_tc<64, true>(a, st) : launch_prefill_tc<64, false>(a, st);
  return -2;
}

}  // namespace barq
