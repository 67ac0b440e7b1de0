// K2: quantized GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), GGUF dequant in the
// mainloop.  out[t, n] = sum_k x[t, k] * W[n, k] for prefill and batched decode.
//
// The reference's quantized matmul is a host round trip (backend/src/cuda_quant.rs:104-126); its
// dense path is a rayon triple loop (barq_core/src/blas.rs:193-207).
//
// Swap-AB tiling: the MMA "A" operand is a 128-row tile of *weights* (dequantized to bf16 on the
// fly), the "B" operand a BN-row tile of *tokens* (bf16 activations), so D = W_tile * X_tile^T sits
// in TMEM as 128 lanes (output features) x BN columns (tokens).  This keeps M = 128 for any token
// count and lets small decode batches (BN = 64) use the same kernel.
//
// Warp roles (320 threads):
//   warps 0-7  dequant: wait for the quantized planes of stage s in shared memory (TMA), expand
//              them to bf16 directly in the UMMA 128B-swizzle K-major layout, fence the async proxy,
//              signal "A full"; after the mainloop they run the epilogue (tcgen05.ld -> global).
//   warp 8     TMA producer: quantized weight planes and the activation tile of every stage.
//   warp 9     MMA issuer: one elected thread issues 4 x tcgen05.mma (K = 16) per 64-wide stage and
//              commits each stage's completion to the stage's "consumed" mbarrier.
// Every wait is bounded (tc_common.cuh); on expiry the CTA records an error word and unwinds.
// No TMA load here uses .multicast::cluster.
#include <cudaTypedefs.h>

#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "gemv_traits.cuh"
#include "launch.h"
#include "tc_common.cuh"

namespace barq {

using namespace tc;

struct GemmDev {
  int N, K, T;
  const uint16_t* d;  // per-block f16 scale plane (Q4_0 / IQ4_NL / Q8_0 / Q6_K)
  int mode;
  float* out_f32;
  __nv_bfloat16* out_bf16;
  const float* bias;
  int ld_out;
  int k_splits;
  int* err;
};

// Staging box widths (bytes per weight row per 64-wide K stage) and x-coordinate rule per plane.
template <int WT> struct Planes;
template <> struct Planes<W_Q4_K> {
  static constexpr int w0 = 32, w1 = 0, w2 = 16;
  static BARQ_DEV int x0(int s) { return 32 * s; }
  static BARQ_DEV int x1(int) { return 0; }
  static BARQ_DEV int x2(int s) { return 16 * (s >> 2); }
};
template <> struct Planes<W_Q5_K> {
  static constexpr int w0 = 32, w1 = 32, w2 = 16;
  static BARQ_DEV int x0(int s) { return 32 * s; }
  static BARQ_DEV int x1(int s) { return 32 * (s >> 2); }
  static BARQ_DEV int x2(int s) { return 16 * (s >> 2); }
};
template <> struct Planes<W_Q6_K> {
  static constexpr int w0 = 64, w1 = 32, w2 = 16;
  static BARQ_DEV int x0(int s) { return 64 * (s >> 1); }
  static BARQ_DEV int x1(int s) { return 32 * (s >> 1); }
  static BARQ_DEV int x2(int s) { return 16 * (s >> 2); }
};
template <> struct Planes<W_Q8_0> {
  static constexpr int w0 = 64, w1 = 0, w2 = 0;
  static BARQ_DEV int x0(int s) { return 64 * s; }
  static BARQ_DEV int x1(int) { return 0; }
  static BARQ_DEV int x2(int) { return 0; }
};
template <> struct Planes<W_Q4_0> {
  static constexpr int w0 = 32, w1 = 0, w2 = 0;
  static BARQ_DEV int x0(int s) { return 32 * s; }
  static BARQ_DEV int x1(int) { return 0; }
  static BARQ_DEV int x2(int) { return 0; }
};
template <> struct Planes<W_IQ4_NL> : Planes<W_Q4_0> {};

// ---- dequantization of one thread's 16 weights (row r, quarter qq of the 64-wide stage s)
//
// Every format is first reduced to four words of unsigned byte codes u (one code per weight, in
// natural element order) plus (zero point zp, scale sc, bias bi) so that  w = (u - zp) * sc + bi.
// fp16 operands: a byte permute places two codes in the mantissas of 1024.0h (exact), one packed
// subtract removes 1024 + zp, one packed FMA applies scale and bias: ~2 instructions per weight.
// bf16 operands: the same codes go through fp32 (mantissa of 2^23, subtract, FMA) and a packed
// round to bf16x2.
struct Codes {
  uint32_t u[4];
  float zp, sc, bi;
};

template <int WT>
BARQ_DEV Codes load_codes(const uint8_t* st0, const uint8_t* st1, const uint8_t* st2, int r, int qq, int s,
                          int grow, const GemmDev& g) {
  Codes c;
  if constexpr (WT == W_Q4_K || WT == W_Q5_K) {
    const int j = s & 3, h = qq >> 1, l0 = 16 * (qq & 1);
    uint4 q = *reinterpret_cast<const uint4*>(st0 + r * 32 + l0);
    uint4 hd = *reinterpret_cast<const uint4*>(st2 + r * 16);
    int scl, mn;
    kscale(hd.y, hd.z, hd.w, 2 * j + h, scl, mn);
    c.sc = h2f(hd.x & 0xFFFF) * (float)scl;
    c.bi = -h2f(hd.x >> 16) * (float)mn;
    c.zp = 0.f;
    uint32_t w[4] = {q.x, q.y, q.z, q.w};
    uint32_t hb[4] = {0, 0, 0, 0};
    if constexpr (WT == W_Q5_K) {
      uint4 qh = *reinterpret_cast<const uint4*>(st1 + r * 32 + l0);
      hb[0] = qh.x; hb[1] = qh.y; hb[2] = qh.z; hb[3] = qh.w;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t v = (h ? (w[i] >> 4) : w[i]) & 0x0F0F0F0Fu;
      if constexpr (WT == W_Q5_K) v |= ((hb[i] >> (2 * j + h)) & 0x01010101u) << 4;
      c.u[i] = v;
    }
  } else if constexpr (WT == W_Q6_K) {
    const int c4 = s & 3, n = c4 >> 1, hh = c4 & 1, qd = 2 * hh + (qq >> 1), l0 = 16 * (qq & 1);
    uint4 ql = *reinterpret_cast<const uint4*>(st0 + r * 64 + ((qd & 1) ? 32 : 0) + l0);
    uint4 qh = *reinterpret_cast<const uint4*>(st1 + r * 32 + l0);
    const int8_t scl = reinterpret_cast<const int8_t*>(st2 + r * 16)[8 * n + 2 * qd + (l0 >> 4)];
    const float dd = grow < g.N ? h2f(g.d[(size_t)grow * (g.K / 256) + (s >> 2)]) : 0.f;
    c.sc = dd * (float)scl;
    c.bi = 0.f;
    c.zp = 32.f;
    uint32_t w[4] = {ql.x, ql.y, ql.z, ql.w}, hb[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      c.u[i] = ((qd >= 2 ? (w[i] >> 4) : w[i]) & 0x0F0F0F0Fu) | (((hb[i] >> (2 * qd)) & 0x03030303u) << 4);
  } else if constexpr (WT == W_Q8_0) {
    const int blk = qq >> 1;
    uint4 q = *reinterpret_cast<const uint4*>(st0 + r * 64 + 32 * blk + 16 * (qq & 1));
    c.sc = grow < g.N ? h2f(g.d[(size_t)grow * (g.K / 32) + 2 * s + blk]) : 0.f;
    c.bi = 0.f;
    c.zp = 128.f;
    c.u[0] = q.x ^ 0x80808080u; c.u[1] = q.y ^ 0x80808080u; c.u[2] = q.z ^ 0x80808080u; c.u[3] = q.w ^ 0x80808080u;
  } else {  // Q4_0 / IQ4_NL: block 2s + qq/2; qq&1 selects low (elements 0-15) or high nibbles (16-31)
    const int blk = qq >> 1, hi = qq & 1;
    uint4 q = *reinterpret_cast<const uint4*>(st0 + r * 32 + 16 * blk);
    c.sc = grow < g.N ? h2f(g.d[(size_t)grow * (g.K / 32) + 2 * s + blk]) : 0.f;
    c.bi = 0.f;
    uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t v = (hi ? (w[i] >> 4) : w[i]) & 0x0F0F0F0Fu;
      if constexpr (WT == W_IQ4_NL) {
        const int t0 = 0xBFAD9881, t1 = 0xF6EADDCF, t2 = 0x26190D01, t3 = 0x71594535;
        v = (uint32_t)lut16((int)v, t0, t1, t2, t3) ^ 0x80808080u;
      }
      c.u[i] = v;
    }
    c.zp = WT == W_IQ4_NL ? 128.f : 8.f;
  }
  return c;
}

// 16 codes -> two 16-byte chunks of fp16 (F16 = true) or bf16 operands.
template <bool F16>
BARQ_DEV void codes_to_operands(const Codes& c, uint4* out) {
  uint32_t r[8];
  if constexpr (F16) {
    const __half2 off = __float2half2_rn(1024.f + c.zp);
    const __half2 sc = __float2half2_rn(c.sc);
    const __half2 bi = __float2half2_rn(c.bi);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t p0 = __byte_perm(c.u[i], 0x64646464u, 0x4140);  // (1024 + u0, 1024 + u1)
      uint32_t p1 = __byte_perm(c.u[i], 0x64646464u, 0x4342);  // (1024 + u2, 1024 + u3)
      __half2 h0 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&p0), off), sc, bi);
      __half2 h1 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&p1), off), sc, bi);
      r[2 * i] = *reinterpret_cast<uint32_t*>(&h0);
      r[2 * i + 1] = *reinterpret_cast<uint32_t*>(&h1);
    }
  } else {
    const float off = 8388608.0f + c.zp;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float f[4];
#pragma unroll
      for (int k = 0; k < 4; ++k)
        f[k] = fmaf(__uint_as_float(__byte_perm(c.u[i], 0x4B000000u, 0x7650 + k)) - off, c.sc, c.bi);
      __nv_bfloat162 b0 = __floats2bfloat162_rn(f[0], f[1]), b1 = __floats2bfloat162_rn(f[2], f[3]);
      r[2 * i] = *reinterpret_cast<uint32_t*>(&b0);
      r[2 * i + 1] = *reinterpret_cast<uint32_t*>(&b1);
    }
  }
  out[0] = make_uint4(r[0], r[1], r[2], r[3]);
  out[1] = make_uint4(r[4], r[5], r[6], r[7]);
}

template <int WT, int BN, int S>
struct GemmSmem {
  static constexpr int A_BYTES = 128 * 128;       // 128 rows x 64 fp16/bf16
  static constexpr int B_BYTES = BN * 128;        // BN rows x 64 fp16/bf16
  static constexpr int QW0 = Planes<WT>::w0 * 128, QW1 = Planes<WT>::w1 * 128, QW2 = Planes<WT>::w2 * 128;
  static constexpr int Q_BYTES = QW0 + QW1 + QW2;
  static constexpr int XCH_BYTES = 4 * 32 * 32 * 4;  // SwiGLU gate/up exchange, one 32x32 f32 tile per quadrant
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + S * A_BYTES;
  static constexpr int OFF_Q = OFF_B + S * B_BYTES;
  static constexpr int OFF_XCH = OFF_Q + S * Q_BYTES;
  static constexpr int OFF_BAR = OFF_XCH + XCH_BYTES;
  static constexpr int N_BAR = 5 * S + 4;
  static constexpr int OFF_TMEM = OFF_BAR + N_BAR * 8;
  static constexpr int TOTAL = OFF_TMEM + 16 + 1024;  // + alignment slack
};

// Warp roles of the persistent kernel.
constexpr int kDequantWarps = 16;  // 4 per TMEM lane quadrant; each thread expands 16 weights per stage
constexpr int kEpiWarp0 = kDequantWarps;      // 4 epilogue warps, one per lane quadrant
constexpr int kTmaWarp = kDequantWarps + 4;
constexpr int kMmaWarp = kDequantWarps + 5;
constexpr int kThreads = (kDequantWarps + 6) * 32;

struct TileMap {
  int n_tiles, t_tiles, ks, total;
  BARQ_DEV void decode(int u, int& nt, int& tt, int& z) const {
    nt = u % n_tiles;  // weight tiles fastest: concurrent CTAs share one activation tile in L2
    const int rest = u / n_tiles;
    z = rest % ks;
    tt = rest / ks;
  }
};

// Persistent: one CTA per SM walks tiles blockIdx.x, +gridDim.x, ...  The smem ring (S stages) and
// the stage counter run continuously across tiles; the accumulator is double-buffered in TMEM
// (2 x BN columns) so the epilogue of one tile overlaps the mainloop of the next.
template <int WT, int BN, int S, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap tx, const __grid_constant__ CUtensorMap tp0,
                    const __grid_constant__ CUtensorMap tp1, const __grid_constant__ CUtensorMap tp2, GemmDev g) {
  using L = GemmSmem<WT, BN, S>;
  using P = Planes<WT>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* fullQ = bars;
  uint64_t* emptyQ = bars + S;
  uint64_t* fullB = bars + 2 * S;
  uint64_t* fullA = bars + 3 * S;
  uint64_t* consumed = bars + 4 * S;
  uint64_t* accFull = bars + 5 * S;      // [2]
  uint64_t* accEmpty = bars + 5 * S + 2; // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_TMEM);
  __shared__ int err_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  TileMap tm;
  tm.n_tiles = (g.N + 127) / 128;
  tm.t_tiles = (g.T + BN - 1) / BN;
  tm.ks = g.k_splits;
  tm.total = tm.n_tiles * tm.t_tiles * tm.ks;
  const int nst_total = g.K / 64;
  auto krange = [&](int z, int& kb, int& ke) {
    kb = (int)((long)nst_total * z / g.k_splits);
    ke = (int)((long)nst_total * (z + 1) / g.k_splits);
  };

  if (threadIdx.x == 0) {
    err_s = 0;
    for (int i = 0; i < S; ++i) {
      mbar_init(&fullQ[i], 1);
      mbar_init(&emptyQ[i], kDequantWarps);
      mbar_init(&fullB[i], 1);
      mbar_init(&fullA[i], kDequantWarps);
      mbar_init(&consumed[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accFull[b], 1);
      mbar_init(&accEmpty[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  volatile int* err = &err_s;

  if (warp == kTmaWarp) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&tx);
      prefetch_tmap(&tp0);
      if (P::w1) prefetch_tmap(&tp1);
      if (P::w2) prefetch_tmap(&tp2);
      int it = 0;
      for (int u = blockIdx.x; u < tm.total && !*err; u += gridDim.x) {
        int nt, tt, z, kb, ke;
        tm.decode(u, nt, tt, z);
        krange(z, kb, ke);
        for (int ks = kb; ks < ke; ++ks, ++it) {
          const int s = it % S, ph = (it / S) & 1;
          if (it >= S && !mbar_wait(&emptyQ[s], ph ^ 1, err, 1)) break;
          uint8_t* q = smem + L::OFF_Q + s * L::Q_BYTES;
          mbar_expect_tx(&fullQ[s], L::Q_BYTES);
          tma_load_2d(q, &tp0, P::x0(ks), nt * 128, &fullQ[s]);
          if (P::w1) tma_load_2d(q + L::QW0, &tp1, P::x1(ks), nt * 128, &fullQ[s]);
          if (P::w2) tma_load_2d(q + L::QW0 + L::QW1, &tp2, P::x2(ks), nt * 128, &fullQ[s]);
          if (it >= S && !mbar_wait(&consumed[s], ph ^ 1, err, 2)) break;
          mbar_expect_tx(&fullB[s], L::B_BYTES);
          tma_load_2d(smem + L::OFF_B + s * L::B_BYTES, &tx, 64 * ks, tt * BN, &fullB[s]);
        }
      }
    }
  } else if (warp == kMmaWarp) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = F16 ? idesc_f16(128, BN) : idesc_bf16(128, BN);
      int it = 0, tc = 0;
      for (int u = blockIdx.x; u < tm.total && !*err; u += gridDim.x, ++tc) {
        int nt, tt, z, kb, ke;
        tm.decode(u, nt, tt, z);
        krange(z, kb, ke);
        const int buf = tc & 1, use = tc >> 1;
        if (tc >= 2 && !mbar_wait(&accEmpty[buf], (use - 1) & 1, err, 8)) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * BN);
        bool ok = true;
        for (int ks = kb; ks < ke; ++ks, ++it) {
          const int s = it % S, ph = (it / S) & 1;
          if (!mbar_wait(&fullA[s], ph, err, 3) || !mbar_wait(&fullB[s], ph, err, 4)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a0 = smem_addr(smem + L::OFF_A + s * L::A_BYTES);
          const uint32_t b0 = smem_addr(smem + L::OFF_B + s * L::B_BYTES);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            mma_bf16(acc, umma_desc_sw128(a0 + 32 * k), umma_desc_sw128(b0 + 32 * k), idesc, (ks > kb) | (k > 0));
          mma_commit(&consumed[s]);
        }
        if (!ok) break;
        mma_commit(&accFull[buf]);
      }
    }
  } else if (warp < kDequantWarps) {
    // ---------------------------------------------------------------- dequant producers
    const int quad = warp & 3, qq = warp >> 2;
    const int r = quad * 32 + lane;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < tm.total && ok && !*err; u += gridDim.x) {
      int nt, tt, z, kb, ke;
      tm.decode(u, nt, tt, z);
      krange(z, kb, ke);
      const int grow = nt * 128 + r;
      for (int ks = kb; ks < ke; ++ks, ++it) {
        const int s = it % S, ph = (it / S) & 1;
        if (!mbar_wait(&fullQ[s], ph, err, 5)) {
          ok = false;
          break;
        }
        const uint8_t* q = smem + L::OFF_Q + s * L::Q_BYTES;
        const Codes cd = load_codes<WT>(q, q + L::QW0, q + L::QW0 + L::QW1, r, qq, ks, grow, g);
        __syncwarp();
        if (lane == 0) mbar_arrive(&emptyQ[s]);
        uint4 ops[2];
        codes_to_operands<F16>(cd, ops);
        if (it >= S && !mbar_wait(&consumed[s], ph ^ 1, err, 6)) {
          ok = false;
          break;
        }
        uint8_t* arow = smem + L::OFF_A + s * L::A_BYTES + r * 128;
        *reinterpret_cast<uint4*>(arow + (((2 * qq) ^ (r & 7)) << 4)) = ops[0];
        *reinterpret_cast<uint4*>(arow + (((2 * qq + 1) ^ (r & 7)) << 4)) = ops[1];
        fence_proxy_async();
        __syncwarp();
        if (lane == 0) mbar_arrive(&fullA[s]);
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (4 warps)
    const int quad = warp - kEpiWarp0;
    const int r = quad * 32 + lane;
    using AT = typename std::conditional<F16, __half, __nv_bfloat16>::type;
    AT* out_act = reinterpret_cast<AT*>(g.out_bf16);
    float* xch = reinterpret_cast<float*>(smem + L::OFF_XCH);
    const bool atomic = g.k_splits > 1;
    int tc = 0;
    for (int u = blockIdx.x; u < tm.total; u += gridDim.x, ++tc) {
      int nt, tt, z;
      tm.decode(u, nt, tt, z);
      const int buf = tc & 1, use = tc >> 1;
      mbar_wait(&accFull[buf], use & 1, err, 7);
      tc_fence_after();
      // All 128 epilogue threads agree on `stop` (the error word only grows).
      asm volatile("bar.sync 2, 128;" ::: "memory");
      if (*err) break;
      const int n0 = nt * 128, t0 = tt * BN, n = n0 + r;
      const uint32_t acc = tmem + (uint32_t)(buf * BN) + ((uint32_t)(quad * 32) << 16);
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld32(acc + (uint32_t)c0, v);
        if (g.mode == EPI_SWIGLU_Q8) {
          // rows [32 gate | 32 up] x 2 groups: quadrants 0,2 hold gate rows, 1,3 the matching up rows
          float* mine = xch + quad * 32 * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) mine[j * 32 + lane] = v[j];
          asm volatile("bar.sync 2, 128;" ::: "memory");
          if ((quad & 1) == 0) {
            const float* up = xch + (quad + 1) * 32 * 32;
            const int f = n0 / 2 + (quad >> 1) * 32 + lane;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int t = t0 + c0 + j;
              if (t < g.T && f < g.N / 2)
                out_act[(size_t)t * g.ld_out + f] = from_f<AT>(silu(v[j]) * up[j * 32 + lane]);
            }
          }
          asm volatile("bar.sync 2, 128;" ::: "memory");
          continue;
        }
        if (n < g.N) {
          const float bias = (g.bias && z == 0) ? g.bias[n] : 0.f;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int t = t0 + c0 + j;
            if (t >= g.T) continue;
            const size_t idx = (size_t)t * g.ld_out + n;
            const float val = v[j] + bias;
            if (g.mode == EPI_STORE_BF16) {
              out_act[idx] = from_f<AT>(val);
            } else if (atomic) {
              atomicAdd(g.out_f32 + idx, val);
            } else if (g.mode == EPI_ADD_F32) {
              g.out_f32[idx] += val;
            } else {
              g.out_f32[idx] = val;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&accEmpty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * BN);
  }
  if (threadIdx.x == 0 && err_s && g.err) atomicExch(g.err, err_s);
}

// ------------------------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
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

static int make_map_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                       uint64_t outer, uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
                       CUtensorMapSwizzle sw) {
  auto enc = get_encode();
  if (!enc) return -10;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t es[2] = {1, 1};
  (void)elem_bytes;
  CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -11;
}

static int* device_err_word() {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static std::unordered_map<int, int*> words;
  std::lock_guard<std::mutex> lk(mu);
  auto it = words.find(dev);
  if (it != words.end()) return it->second;
  int* p = nullptr;
  if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
  cudaMemset(p, 0, sizeof(int));
  words[dev] = p;
  return p;
}

int gemm_error_word(int* host_out) {
  int* p = device_err_word();
  if (!p) return -1;
  return cudaMemcpy(host_out, p, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -1;
}

int gemm_clear_error_word() {
  int* p = device_err_word();
  return p && cudaMemset(p, 0, sizeof(int)) == cudaSuccess ? 0 : -1;
}

template <int WT, int BN, int S, bool F16>
static int launch_gemm(const QW& w, const CUtensorMap& tx, const CUtensorMap& m0, const CUtensorMap& m1,
                       const CUtensorMap& m2, const GemmDev& g, int tiles_t, cudaStream_t st) {
  using L = GemmSmem<WT, BN, S>;
  static_assert(L::TOTAL <= 232448, "shared memory budget");
  auto kern = qgemm_tc_kernel<WT, BN, S, F16>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
  const int total = ((w.N + 127) / 128) * tiles_t * g.k_splits;
  static int n_sm = 0;
  if (!n_sm) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev);
    if (n_sm <= 0) n_sm = 148;
  }
  dim3 grid(total < n_sm ? total : n_sm);
  kern<<<grid, kThreads, L::TOTAL, st>>>(tx, m0, m1, m2, g);
  return cudaPeekAtLastError() == cudaSuccess ? 0 : -20;
}

template <int WT, bool F16>
static int dispatch_bn(const QW& w, const void* x, int T, const GemmDev& g0, cudaStream_t st) {
  using P = Planes<WT>;
  GemmDev g = g0;
  const int K = w.K, N = w.N;
  CUtensorMap mx, m0, m1, m2;
  memset(&m1, 0, sizeof(m1));
  memset(&m2, 0, sizeof(m2));
  int bn = T <= 64 ? 64 : (T <= 128 ? 128 : 256);
  int rc = make_map_2d(&mx, x, F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, K, T,
                       (uint64_t)K * 2, 64, bn, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  uint64_t rb0 = WT == W_Q8_0 ? K : (WT == W_Q6_K ? K / 2 : K / 2);
  rc = make_map_2d(&m0, w.p0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rb0, N, rb0, P::w0, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  if (P::w1) {
    uint64_t rb1 = WT == W_Q5_K ? K / 8 : K / 4;
    rc = make_map_2d(&m1, w.p1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rb1, N, rb1, P::w1, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  if (P::w2) {
    uint64_t rb2 = WT == W_Q6_K ? K / 16 : (K / 256) * 16;
    rc = make_map_2d(&m2, w.p2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, rb2, N, rb2, P::w2, 128, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  const int tiles_t = (T + bn - 1) / bn;
  if (g.k_splits == 0) {  // auto split-K so that small token counts still fill the 148 SMs
    const int tiles = ((N + 127) / 128) * tiles_t, nst = K / 64;
    int ks = 1;
    if (g.mode == EPI_STORE_F32 || g.mode == EPI_ADD_F32)
      while (tiles * ks * 2 <= 2 * 148 && nst / (ks * 2) >= 4) ks *= 2;
    g.k_splits = ks;
  }
  if (g.k_splits > 1 && g.mode == EPI_STORE_F32) {
    if (cudaMemset2DAsync(g.out_f32, (size_t)g.ld_out * 4, 0, (size_t)N * 4, T, st) != cudaSuccess) return -6;
  }
  if (bn == 64) return launch_gemm<WT, 64, 5, F16>(w, mx, m0, m1, m2, g, tiles_t, st);
  if (bn == 128) return launch_gemm<WT, 128, 4, F16>(w, mx, m0, m1, m2, g, tiles_t, st);
  return launch_gemm<WT, 256, 3, F16>(w, mx, m0, m1, m2, g, tiles_t, st);
}

template <bool F16>
static int dispatch_type(const QW& w, const void* x, int T, const GemmDev& g, cudaStream_t st) {
  switch (w.type) {
    case W_Q4_K: return dispatch_bn<W_Q4_K, F16>(w, x, T, g, st);
    case W_Q5_K: return dispatch_bn<W_Q5_K, F16>(w, x, T, g, st);
    case W_Q6_K: return dispatch_bn<W_Q6_K, F16>(w, x, T, g, st);
    case W_Q8_0: return dispatch_bn<W_Q8_0, F16>(w, x, T, g, st);
    case W_Q4_0: return dispatch_bn<W_Q4_0, F16>(w, x, T, g, st);
    case W_IQ4_NL: return dispatch_bn<W_IQ4_NL, F16>(w, x, T, g, st);
  }
  return -7;
}

int qgemm_tc(const QW& w, const void* x, int x_is_f16, int T, const GemvEpi& ep, int k_splits, cudaStream_t st) {
  if (T <= 0) return 0;
  if (w.K % 256 && !(w.K % 64 == 0 && (w.type == W_Q8_0 || w.type == W_Q4_0 || w.type == W_IQ4_NL))) return -2;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (w.K * 2) % 16) return -3;
  if (ep.mode == EPI_SWIGLU_Q8 && (w.N % 128 || k_splits > 1)) return -4;
  if (ep.mode == EPI_SWIGLU_Q8 || ep.mode == EPI_STORE_BF16) k_splits = 1;
  if (k_splits < 0) k_splits = 0;
  GemmDev g;
  g.N = w.N;
  g.K = w.K;
  g.T = T;
  g.d = w.d;
  g.mode = ep.mode;
  g.out_f32 = ep.out_f32;
  g.out_bf16 = ep.out_bf16;
  g.bias = ep.bias;
  g.ld_out = ep.ld_out;
  g.k_splits = k_splits;
  g.err = device_err_word();
  return x_is_f16 ? dispatch_type<true>(w, x, T, g, st) : dispatch_type<false>(w, x, T, g, st);
}

}  // namespace barq
