// K2: quantized GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), GGUF dequant in the
// mainloop.  out[t, n] = sum_k x[t, k] * W[n, k] for prefill and batched decode.
//
// The reference's quantized matmul is a host round trip (backend/src/cuda_quant.rs:104-126); its
// dense path is a rayon triple loop (barq_core/src/blas.rs:193-207).
//
// Swap-AB tiling: the MMA "A" operand is a 128-row tile of *weights* (dequantized on the fly), the
// "B" operand a BN-row tile of *tokens* (fp16/bf16 activations), so D = W_tile * X_tile^T sits in
// TMEM as 128 lanes (output features) x BN columns (tokens).  M = 128 for any token count, so small
// decode batches (BN = 64) and prefill (BN = 256) share the kernel.
//
// Data movement: weights are stored tiled (qtile.cuh), so the quantized planes of one 128-row x
// G-column group are one contiguous chunk fetched with a single cp.async.bulk; activations arrive
// as 128-byte-swizzled TMA tiles.  Persistent: one CTA per SM walks the tile list; the smem rings
// and their stage counters run continuously across tiles, and the accumulator is double-buffered in
// TMEM (2 x BN columns) so the epilogue of one tile overlaps the mainloop of the next.
//
// Warp roles (736 threads):
//   warps 0-15  dequant: expand 16 weights each per 64-column stage straight into the UMMA
//               128B-swizzle K-major layout, fence the async proxy, signal "A full";
//   warps 16-19 epilogue: tcgen05.ld the finished accumulator -> global (store / residual add /
//               split-K atomics / SwiGLU);
//   warp 20     weight producer: bulk copies of weight chunks, up to SQ chunks ahead;
//   warp 21     activation producer: TMA of activation tiles, one ring slot behind the MMAs;
//   warp 22     MMA: one thread issues 4 x tcgen05.mma (K = 16) per stage and commits completion.
// Every wait is bounded (tc_common.cuh); on expiry the CTA records an error word and unwinds.
// Every TMA / bulk copy here has a single destination CTA and reads this GPU's own memory.
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>
#include <type_traits>
#include <unordered_map>

#include "gemv_traits.cuh"
#include "launch.h"
#include "pdl.cuh"
#include "qtile.cuh"
#include "sysflags.cuh"
#include "tc_common.cuh"

namespace barq {

using namespace tc;

struct GemmDev {
  int N, K, T;
  const uint8_t* w;  // tiled weight chunks
  int mode;
  float* out_f32;
  void* out_act;
  const float* bias;
  int ld_out;
  int k_splits;
  int* err;
  // Grouped (MoE) mode, ng > 0: the weight holds ng groups of grows rows (one expert each); the
  // activation rows are sorted by group, group e owning rows [goff[e], goff[e+1]) (device memory,
  // written by the routing kernels).  Output columns are group-local (0..grows).  EPI_MOE_COMBINE
  // adds row_w[row] * result into out_f32[row_tok[row], :] with atomics.
  const int* goff;
  int ng, grows;
  const int* row_tok;
  const float* row_w;
  // Split-K (k_splits > 1): each split stores its partial tile in split_ws; the last split of a
  // tile to arrive (split_cnt, one zeroed counter per output tile) sums them in split order.
  float* split_ws;
  int* split_cnt;
  // Sequence-parallel tensor parallelism: EPI_RS_PUSH target (rs), and the all-gather flags the
  // activation producer waits on before loading a token tile (agw.flags non-null).
  SpPush rs;
  SpWait agw;
  int exp;  // diagnostics (built with BARQ_DIAG): bit 0 = skip the dequant arithmetic (write zeros), bit 1 = trace CTA 0
  unsigned long long* trace;  // [kTraceStages][8] globaltimer stamps when tracing
};
constexpr int kTraceStages = 256;
// trace fields per stage: 0 chunk issued, 1 chunk landed (dequant warp 0), 2 A written (dequant 0),
// 3 act issued, 4 MMA saw A, 5 MMA saw B, 6 MMA issued, 7 consumed observed by dequant 0
BARQ_DEV void trace(const GemmDev& g, int stage, int field) {
  if ((kDiag && (g.exp & 2)) && blockIdx.x == 0 && stage < kTraceStages && g.trace)
    g.trace[stage * 32 + field] = clock64();
}

// 1-D bulk copy global -> shared, completion on `bar` (transaction bytes).
BARQ_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// ---- dequantization of one thread's 16 weights (row r, quarter qq of 64-column stage `sub` of
// the staged chunk).  Every format is reduced to four words of unsigned byte codes u (one per
// weight, natural order) plus (zero point zp, scale sc, bias bi) with  w = (u - zp) * sc + bi.
struct Codes {
  uint32_t u[4];
  float zp, sc, bi;
};

BARQ_DEV void words(uint4 v, uint32_t* w) {
  w[0] = v.x;
  w[1] = v.y;
  w[2] = v.z;
  w[3] = v.w;
}

template <int WT>
BARQ_DEV Codes load_codes(const uint8_t* ch, int r, int qq, int sub) {
  using F = TileFmt<WT>;
  Codes c;
  if constexpr (WT == W_Q4_K || WT == W_Q5_K) {
    const int j = sub, h = qq >> 1;
    uint32_t w[4];
    words(*reinterpret_cast<const uint4*>(staged_chunk<WT, 0>(ch, r, 2 * j + (qq & 1))), w);
    constexpr int HP = WT == W_Q5_K ? 2 : 1;
    const uint4 hd = *reinterpret_cast<const uint4*>(staged_chunk<WT, HP>(ch, r, 0));
    int scl, mn;
    kscale(hd.y, hd.z, hd.w, 2 * j + h, scl, mn);
    c.sc = h2f(hd.x & 0xFFFF) * (float)scl;
    c.bi = -h2f(hd.x >> 16) * (float)mn;
    c.zp = 0.f;
    uint32_t hb[4] = {0, 0, 0, 0};
    if constexpr (WT == W_Q5_K) words(*reinterpret_cast<const uint4*>(staged_chunk<WT, 1>(ch, r, qq & 1)), hb);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t v = (h ? (w[i] >> 4) : w[i]) & 0x0F0F0F0Fu;
      if constexpr (WT == W_Q5_K) v |= ((hb[i] >> (2 * j + h)) & 0x01010101u) << 4;
      c.u[i] = v;
    }
  } else if constexpr (WT == W_Q6_K) {
    const int n = sub >> 1, hh = sub & 1, qd = 2 * hh + (qq >> 1), l0c = qq & 1;
    uint32_t w[4], hb[4];
    words(*reinterpret_cast<const uint4*>(staged_chunk<WT, 0>(ch, r, 4 * n + 2 * (qd & 1) + l0c)), w);
    words(*reinterpret_cast<const uint4*>(staged_chunk<WT, 1>(ch, r, 2 * n + l0c)), hb);
    const int8_t scl = reinterpret_cast<const int8_t*>(staged_chunk<WT, 2>(ch, r, 0))[8 * n + 2 * qd + l0c];
    const float dd = h2f(reinterpret_cast<const uint16_t*>(ch + F::D_OFF)[r]);
    c.sc = dd * (float)scl;
    c.bi = 0.f;
    c.zp = 32.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      c.u[i] = ((qd >= 2 ? (w[i] >> 4) : w[i]) & 0x0F0F0F0Fu) | (((hb[i] >> (2 * qd)) & 0x03030303u) << 4);
  } else if constexpr (WT == W_Q8_0) {
    const int bi = qq >> 1;
    uint32_t w[4];
    words(*reinterpret_cast<const uint4*>(staged_chunk<WT, 0>(ch, r, 2 * bi + (qq & 1))), w);
    c.sc = h2f(reinterpret_cast<const uint16_t*>(ch + F::D_OFF)[2 * r + bi]);
    c.bi = 0.f;
    c.zp = 128.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) c.u[i] = w[i] ^ 0x80808080u;
  } else {  // Q4_0 / IQ4_NL: block qq/2 of the stage; qq&1 selects low (elements 0-15) or high nibbles
    const int bi = qq >> 1, hi = qq & 1;
    uint32_t w[4];
    words(*reinterpret_cast<const uint4*>(staged_chunk<WT, 0>(ch, r, bi)), w);
    c.sc = h2f(reinterpret_cast<const uint16_t*>(ch + F::D_OFF)[2 * r + bi]);
    c.bi = 0.f;
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
// fp16: a byte permute places two codes in the mantissas of 1024.0h (exact), one packed subtract
// removes 1024 + zp, one packed FMA applies scale and bias (~2 instructions per weight).
// bf16: codes go through fp32 (mantissa of 2^23, subtract, FMA) and a packed round to bf16x2.
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

// One 32-weight sub-block (row r; 64-column atom sub64 of the staged chunk; its first or second 32
// columns by h) -> four 16-byte groups of operand pairs.  Q4_K / Q5_K share one (scale, min) over
// the sub-block, decoded once; other formats expand two 16-weight halves.
template <int WT, bool F16>
BARQ_DEV void dequant32(const uint8_t* ch, int r, int sub64, int h, uint4* out) {
  if constexpr ((WT == W_Q4_K || WT == W_Q5_K) && F16) {
    // fp16-native scale: (1024 + scl, 1024) - (1024, 1024 + mn) = (scl, -mn) exactly, times the
    // (d, dmin) pair -> (d*scl, -dmin*mn), each product rounded once, as a float product rounded to
    // fp16 would be; no int/float conversion instructions.
    constexpr int HP = WT == W_Q5_K ? 2 : 1;
    const uint4 hd = *reinterpret_cast<const uint4*>(staged_chunk<WT, HP>(ch, r, 0));
    int scl, mn;
    kscale(hd.y, hd.z, hd.w, 2 * sub64 + h, scl, mn);
    uint32_t ua = 0x64006400u | (uint32_t)scl, ub = 0x64006400u | ((uint32_t)mn << 16);
    const __half2 t = __hsub2(*reinterpret_cast<__half2*>(&ua), *reinterpret_cast<__half2*>(&ub));
    uint32_t dd = hd.x;
    const __half2 sb = __hmul2(*reinterpret_cast<__half2*>(&dd), t);
    const __half2 sc2 = __low2half2(sb), bi2 = __high2half2(sb);
    const __half2 off = __float2half2_rn(1024.f);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t w[4];
      words(*reinterpret_cast<const uint4*>(staged_chunk<WT, 0>(ch, r, 2 * sub64 + half)), w);
      uint32_t hb[4] = {0, 0, 0, 0};
      if constexpr (WT == W_Q5_K) words(*reinterpret_cast<const uint4*>(staged_chunk<WT, 1>(ch, r, half)), hb);
      uint32_t o[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t v = (h ? (w[i] >> 4) : w[i]) & 0x0F0F0F0Fu;
        if constexpr (WT == W_Q5_K) v |= ((hb[i] >> (2 * sub64 + h)) & 0x01010101u) << 4;
        uint32_t p0 = __byte_perm(v, 0x64646464u, 0x4140), p1 = __byte_perm(v, 0x64646464u, 0x4342);
        __half2 h0 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&p0), off), sc2, bi2);
        __half2 h1 = __hfma2(__hsub2(*reinterpret_cast<__half2*>(&p1), off), sc2, bi2);
        o[2 * i] = *reinterpret_cast<uint32_t*>(&h0);
        o[2 * i + 1] = *reinterpret_cast<uint32_t*>(&h1);
      }
      out[2 * half] = make_uint4(o[0], o[1], o[2], o[3]);
      out[2 * half + 1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
  } else if constexpr (WT == W_Q4_K || WT == W_Q5_K) {
    constexpr int HP = WT == W_Q5_K ? 2 : 1;
    const uint4 hd = *reinterpret_cast<const uint4*>(staged_chunk<WT, HP>(ch, r, 0));
    int scl, mn;
    kscale(hd.y, hd.z, hd.w, 2 * sub64 + h, scl, mn);
    Codes c;
    c.sc = h2f(hd.x & 0xFFFF) * (float)scl;
    c.bi = -h2f(hd.x >> 16) * (float)mn;
    c.zp = 0.f;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t w[4];
      words(*reinterpret_cast<const uint4*>(staged_chunk<WT, 0>(ch, r, 2 * sub64 + half)), w);
      uint32_t hb[4] = {0, 0, 0, 0};
      if constexpr (WT == W_Q5_K) words(*reinterpret_cast<const uint4*>(staged_chunk<WT, 1>(ch, r, half)), hb);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t v = (h ? (w[i] >> 4) : w[i]) & 0x0F0F0F0Fu;
        if constexpr (WT == W_Q5_K) v |= ((hb[i] >> (2 * sub64 + h)) & 0x01010101u) << 4;
        c.u[i] = v;
      }
      codes_to_operands<F16>(c, out + 2 * half);
    }
  } else {
    codes_to_operands<F16>(load_codes<WT>(ch, r, 2 * h, sub64), out);
    codes_to_operands<F16>(load_codes<WT>(ch, r, 2 * h + 1, sub64), out + 2);
  }
}

// Whether token tiles of up to 128 rows take the weight operand from TMEM (1) or from shared memory
// (0); see Issuers below.
#ifndef BARQ_GEMM_TS
#define BARQ_GEMM_TS 1
#endif
constexpr bool kGemmTS = BARQ_GEMM_TS != 0;

template <int WT, int BN, int S, int SQ, int KS>
struct GemmSmem {
  static constexpr int A_ATOM = 128 * 128;        // 128 rows x 64 fp16/bf16 (one 128B-swizzle atom column)
  static constexpr int B_ATOM = BN * 128;         // BN rows x 64 fp16/bf16
  static constexpr int A_BYTES = (kGemmTS && BN <= 128) ? 0 : KS * A_ATOM;  // one stage: KS x 64 columns (TS: in TMEM)
  static constexpr int B_BYTES = KS * B_ATOM;
  static constexpr int Q_BYTES = TileFmt<WT>::CHUNK;
  static constexpr int XCH_BYTES = 4 * 32 * 32 * 4;  // SwiGLU exchange, one 32x32 f32 tile per quadrant
  static constexpr int OFF_A = 0;
  static constexpr int OFF_B = OFF_A + S * A_BYTES;
  static constexpr int OFF_Q = OFF_B + S * B_BYTES;
  static constexpr int OFF_XCH = OFF_Q + ((SQ * Q_BYTES + 1023) / 1024) * 1024;
  static constexpr int OFF_BAR = OFF_XCH + XCH_BYTES;
  static constexpr int N_BAR = 2 * SQ + 2 * S + 4;
  static constexpr int OFF_TMEM = OFF_BAR + N_BAR * 8;
  static constexpr int TOTAL = OFF_TMEM + 16 + 1024;  // + alignment slack
};

constexpr int kDequantWarps = 16;  // 4 per TMEM lane quadrant; each thread expands 16 weights per stage
constexpr int kEpiWarp0 = kDequantWarps;  // 4 epilogue warps, one per lane quadrant
constexpr int kTmaWarp = kDequantWarps + 4;  // weight chunks (gated only by chunk-slot release)
constexpr int kActWarp = kDequantWarps + 5;  // activation tiles (gated by MMA progress)
constexpr int kMmaWarp = kDequantWarps + 6;  // MMA issuers: warps kMmaWarp, kMmaWarp + 1
constexpr int kThreads = (kDequantWarps + 8) * 32;
// Two MMA-issuing threads alternate the stages of a tile, each accumulating into its own TMEM
// buffer.  One issuing thread stalls on every tcgen05.mma while the tensor queue is full and then
// pays its per-stage barrier round (commit + wait, a few hundred cycles) with the tensor pipe idle;
// with two, one thread's barrier round overlaps the other's queued MMAs, which keeps M=128 x N<=128
// MMAs near their 64-cycle issue rate.  Wide token tiles (BN = 256) keep one issuer: their MMAs
// already take 128 cycles each and the TMEM budget (512 columns) holds only two 256-column buffers.
//
// Token tiles of up to 128 columns take the weight operand from TMEM ("TS" MMA): dequant warps store
// the expanded weights with tcgen05.st into their own lane quadrant, so the operand never touches
// shared memory (no 32 KB/stage of st.shared, no async-proxy fence, no smem reads by the MMA), and
// the shared memory it frees deepens the activation and weight-chunk rings.  TMEM budget (512
// columns): accumulators 2 buffers x NI issuers x BN, then S stages x KS x 32 columns of operand.
template <int BN>
struct Issuers {
  static constexpr int NI = BN <= 64 ? 2 : 1;
  static constexpr bool TS = kGemmTS && BN <= 128;
  static constexpr int ACOL = 2 * NI * BN;            // first TMEM column of the operand stages
  static constexpr int COLS = TS ? 512 : 2 * NI * BN;
};

constexpr int kMaxGroups = 256;
// Split-K: at most this many K splits per output tile (the last split to finish reads every
// split's partial tile, so more splits lengthen the kernel's tail more than they add parallelism).
constexpr int kMaxAutoSplits = 8;

// One output tile: global weight tile nt, K split z, activation/output rows [row0, row0 + rows),
// output column base n0.
struct Tile {
  int nt, z, row0, rows, n0;
};

template <int BN>
struct TileMap {
  int n_tiles, t_tiles, ks, total, T;
  int ng, ntg;                   // grouped: groups, weight tiles per group
  const int* off;                // [ng+1] activation row offsets (smem)
  const int* tcum;               // [ng+1] prefix of tiles per group (smem)
  BARQ_DEV Tile decode(int u) const {
    Tile t;
    if (ng == 0) {
      t.nt = u % n_tiles;  // weight tiles fastest: concurrent CTAs share one activation tile in L2
      const int rest = u / n_tiles;
      t.z = rest % ks;
      const int tt = rest / ks;
      t.row0 = tt * BN;
      t.rows = min(BN, T - t.row0);
      t.n0 = t.nt * 128;
    } else {
      int e = 0;
      while (tcum[e + 1] <= u) ++e;
      const int local = u - tcum[e], ntl = local % ntg, tt = local / ntg;
      t.nt = e * ntg + ntl;
      t.z = 0;
      t.row0 = off[e] + tt * BN;
      t.rows = min(BN, off[e + 1] - t.row0);
      t.n0 = ntl * 128;
    }
    return t;
  }
};

template <int WT, int BN, int S, int SQ, int KS, bool F16>
__global__ void __launch_bounds__(kThreads, 1)
    qgemm_tc_kernel(const __grid_constant__ CUtensorMap tx, GemmDev g) {
  using L = GemmSmem<WT, BN, S, SQ, KS>;
  using F = TileFmt<WT>;
  static_assert(F::G % (64 * KS) == 0, "a stage never straddles two weight chunks");
  constexpr int SPG = F::G / (64 * KS);  // stages per weight chunk
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* fullQ = bars;                // [SQ] chunk landed
  uint64_t* emptyQ = bars + SQ;          // [SQ] chunk fully expanded
  // full[s]: the stage's weight operand is written (one arrival per dequant warp) AND its activation
  // tile has landed (the producer's arrive.expect_tx + the TMA transaction bytes) -- one barrier, so
  // the MMA thread pays a single wait per stage
  uint64_t* full = bars + 2 * SQ;              // [S]
  uint64_t* consumed = bars + 2 * SQ + S;      // [S] MMAs of the stage done
  uint64_t* accFull = bars + 2 * SQ + 2 * S;   // [2]
  uint64_t* accEmpty = accFull + 2;            // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::OFF_TMEM);
  __shared__ int err_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int goff_s[kMaxGroups + 1], gcum_s[kMaxGroups + 1];
  TileMap<BN> tm;
  tm.n_tiles = (g.N + 127) / 128;
  tm.t_tiles = (g.T + BN - 1) / BN;
  tm.ks = g.k_splits;
  tm.total = tm.n_tiles * tm.t_tiles * tm.ks;
  tm.T = g.T;
  tm.ng = g.ng;
  tm.ntg = g.grows / 128;
  tm.off = goff_s;
  tm.tcum = gcum_s;
  if (g.ng > 0) {
    // Grouped: the group offsets come from the previous kernel, so every role waits for it here.
    pdl_wait();
    for (int i = threadIdx.x; i <= g.ng; i += blockDim.x) goff_s[i] = g.goff[i];
    __syncthreads();
    if (threadIdx.x == 0) {
      int cum = 0;
      for (int e = 0; e < g.ng; ++e) {
        gcum_s[e] = cum;
        cum += (goff_s[e + 1] - goff_s[e] + BN - 1) / BN * tm.ntg;
      }
      gcum_s[g.ng] = cum;
    }
    __syncthreads();
    tm.total = gcum_s[g.ng];
  }
  const int KG = g.K / F::G;
  auto grange = [&](int z, int& gb, int& ge) {
    gb = (int)((long)KG * z / g.k_splits);
    ge = (int)((long)KG * (z + 1) / g.k_splits);
  };

  if (threadIdx.x == 0) {
    err_s = 0;
    for (int i = 0; i < SQ; ++i) {
      mbar_init(&fullQ[i], 1);
      mbar_init(&emptyQ[i], kDequantWarps);
    }
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], kDequantWarps + 1);
      mbar_init(&consumed[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accFull[b], Issuers<BN>::NI);
      mbar_init(&accEmpty[b], 4);
    }
    fence_mbar_init();
  }
  constexpr int NI = Issuers<BN>::NI;
  constexpr bool TS = Issuers<BN>::TS;
  static_assert(!TS || Issuers<BN>::ACOL + S * KS * 32 <= 512, "TMEM budget");
  if (warp == kMmaWarp) tmem_alloc(tmem_slot, Issuers<BN>::COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  volatile int* err = &err_s;
  // Weight chunks, their dequantization and the MMAs on them do not depend on earlier kernels; the
  // activation producer and the epilogue (which writes, or adds into, the output) wait for them.
  pdl_trigger();

  if (warp == kTmaWarp) {
    // ---------------------------------------------------------------- weight-chunk producer
    // Runs up to SQ chunks ahead of the dequant warps, independent of MMA progress.
    if (lane == 0) {
      int qc = 0;
      for (int u = blockIdx.x; u < tm.total && !*err; u += gridDim.x) {
        const Tile tl = tm.decode(u);
        const int nt = tl.nt, z = tl.z;
        int gb, ge;
        grange(z, gb, ge);
        bool ok = true;
        for (int kg = gb; kg < ge; ++kg, ++qc) {
          const int qs = qc % SQ, qph = (qc / SQ) & 1;
          if (qc >= SQ && !mbar_wait(&emptyQ[qs], qph ^ 1, err, 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&fullQ[qs], L::Q_BYTES);
          trace(g, qc * SPG, 0);
          bulk_load(smem + L::OFF_Q + qs * L::Q_BYTES, g.w + ((size_t)nt * KG + kg) * F::CHUNK, L::Q_BYTES,
                    &fullQ[qs]);
        }
        if (!ok) break;
      }
    }
  } else if (warp == kActWarp) {
    // ---------------------------------------------------------------- activation-tile producer
    pdl_wait();
    const uint32_t ag_ep = g.agw.flags ? *g.agw.epoch : 0u;
    int ag_row = 0;  // rows [0, ag_row) of the gathered activation are known to have arrived
    if (lane == 0) prefetch_tmap(&tx);
    int it = 0;
    for (int u = blockIdx.x; u < tm.total; u += gridDim.x) {
      if (__shfl_sync(0xffffffffu, *err != 0, 0)) break;  // warp-uniform stop
      const Tile tl = tm.decode(u);
      const int z = tl.z;
      int gb, ge;
      grange(z, gb, ge);
      bool ok = true;
      if (g.agw.flags && tl.row0 + tl.rows > ag_row) {
        // all-gather consumer: the warp polls the row flags of this token tile (written by the
        // owners' reduce kernels over NVLink), then orders the async proxy (TMA) after them
        bool arrived = true;
        for (int rr = tl.row0 + lane; rr < tl.row0 + tl.rows; rr += 32)
          arrived = arrived && wait_epoch_sys(g.agw.flags + rr, ag_ep, g.agw.wait_ns);
        arrived = __all_sync(0xffffffffu, arrived);
        // A peer that never delivered: record it in the global error word (the host raises) but
        // finish the tile on whatever the buffer holds, so the kernel takes no early-exit path with
        // copies in flight.
        if (!arrived && lane == 0 && g.err) atomicExch(g.err, 0x400);
        asm volatile("fence.proxy.async.global;" ::: "memory");
        ag_row = tl.row0 + tl.rows;  // token tiles of a CTA come in non-decreasing row order
      }
      if (lane == 0) {
        for (int ks = gb * SPG; ks < ge * SPG; ++ks, ++it) {
          const int s = it % S, ph = (it / S) & 1;
          if (it >= S && !mbar_wait(&consumed[s], ph ^ 1, err, 2)) {
            ok = false;
            break;
          }
          trace(g, it, 3);
          if (kDiag && (g.exp & 8)) {  // diagnostics: no activation copy (operand stale), barrier protocol unchanged
            mbar_arrive(&full[s]);
          } else {
            mbar_expect_tx(&full[s], L::B_BYTES);
#pragma unroll
            for (int a = 0; a < KS; ++a)
              tma_load_2d(smem + L::OFF_B + s * L::B_BYTES + a * L::B_ATOM, &tx, 64 * (ks * KS + a), tl.row0, &full[s]);
          }
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
    }
  } else if (warp >= kMmaWarp && warp < kMmaWarp + NI) {
    // ---------------------------------------------------------------- MMA issuers
    // Issuer m takes the stages i of each tile with i % NI == m, accumulating into TMEM columns
    // [(buf * NI + m) * BN, +BN).  It walks every stage to keep the ring index and phase in step.
    const int me = warp - kMmaWarp;
    if (lane == 0) {
      constexpr uint32_t idesc = F16 ? idesc_f16(128, BN) : idesc_bf16(128, BN);
      int it = 0, tc = 0;
      for (int u = blockIdx.x; u < tm.total && !*err; u += gridDim.x, ++tc) {
        const Tile tl = tm.decode(u);
        const int nt = tl.nt, z = tl.z;
        int gb, ge;
        grange(z, gb, ge);
        const int buf = tc & 1, use = tc >> 1;
        const int nst = (ge - gb) * SPG;
        if (tc >= 2 && !mbar_wait(&accEmpty[buf], (use - 1) & 1, err, 8)) break;
        tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)((buf * NI + me) * BN);
        bool ok = true;
        for (int i = 0; i < nst; ++i, ++it) {
          if (i % NI != me) continue;
          const int s = it % S, ph = (it / S) & 1;
          trace(g, it, 0);
          if (!mbar_wait(&full[s], ph, err, 3)) {
            ok = false;
            break;
          }
          trace(g, it, 4);
          tc_fence_after();
          const uint32_t b0 = smem_addr(smem + L::OFF_B + s * L::B_BYTES);
          if constexpr (TS) {
            const uint32_t ta = tmem + (uint32_t)(Issuers<BN>::ACOL + s * KS * 32);
#pragma unroll
            for (int a = 0; a < KS; ++a)
#pragma unroll
              for (int k = 0; k < 4; ++k)
                mma_f16_ts(acc, ta + (uint32_t)(a * 32 + k * 8), umma_desc_sw128(b0 + a * L::B_ATOM + 32 * k), idesc,
                           (i >= NI) | a | k);
          } else {
            const uint32_t a0 = smem_addr(smem + L::OFF_A + s * L::A_BYTES);
#pragma unroll
            for (int a = 0; a < KS; ++a)
#pragma unroll
              for (int k = 0; k < 4; ++k)
                mma_bf16(acc, umma_desc_sw128(a0 + a * L::A_ATOM + 32 * k),
                         umma_desc_sw128(b0 + a * L::B_ATOM + 32 * k), idesc, (i >= NI) | a | k);
          }
          trace(g, it, 1);
          mma_commit(&consumed[s]);
          trace(g, it, 6);
        }
        if (!ok) break;
        mma_commit(&accFull[buf]);  // every issuer arrives, also one that had no stage in this tile
      }
    }
  } else if (warp < kDequantWarps) {
    // ---------------------------------------------------------------- dequant producers
    const int quad = warp & 3, qq = warp >> 2;
    const int r = quad * 32 + lane;
    int it = 0, qc = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < tm.total && ok && !*err; u += gridDim.x) {
      const Tile tl = tm.decode(u);
      const int nt = tl.nt, z = tl.z;
      int gb, ge;
      grange(z, gb, ge);
      for (int kg = gb; kg < ge && ok; ++kg, ++qc) {
        const int qs = qc % SQ, qph = (qc / SQ) & 1;
        if (!mbar_wait(&fullQ[qs], qph, err, 5)) {
          ok = false;
          break;
        }

        const uint8_t* ch = smem + L::OFF_Q + qs * L::Q_BYTES;
        if constexpr (TS && KS == 2) {
          // 128-column stages: warp (quad, sb) expands rows quad*32 + lane, stage columns [32 sb, +32)
#pragma unroll
          for (int sub = 0; sub < SPG; ++sub, ++it) {
            const int s = it % S, ph = (it / S) & 1;
            uint4 ops[4];
            if (kDiag && (g.exp & 1)) {
              ops[0] = ops[1] = ops[2] = ops[3] = make_uint4(0, 0, 0, 0);
            } else {
              dequant32<WT, F16>(ch, r, 2 * sub + (qq >> 1), qq & 1, ops);
            }
            if (it >= S && !mbar_wait(&consumed[s], ph ^ 1, err, 6)) {
              ok = false;
              break;
            }
            if (warp == 0 && lane == 0) trace(g, it, 7);
            tmem_st16(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(Issuers<BN>::ACOL + s * 64 + qq * 16), ops);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full[s]);
            if (warp == 0 && lane == 0) trace(g, it, 2);
          }
          __syncwarp();
          if (ok && lane == 0) mbar_arrive(&emptyQ[qs]);
        } else {
        for (int sub = 0; sub < SPG; ++sub, ++it) {
          const int s = it % S, ph = (it / S) & 1;
          uint4 ops[KS][2];
#pragma unroll
          for (int a = 0; a < KS; ++a) {
            if (kDiag && (g.exp & 1)) {
              ops[a][0] = ops[a][1] = make_uint4(0, 0, 0, 0);
            } else {
              const Codes cd = load_codes<WT>(ch, r, qq, sub * KS + a);
              codes_to_operands<F16>(cd, ops[a]);
            }
          }
          if (it >= S && !mbar_wait(&consumed[s], ph ^ 1, err, 6)) {
            ok = false;
            break;
          }
          if (warp == 0 && lane == 0) trace(g, it, 7);
          if constexpr (TS) {
            const uint32_t ta = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(Issuers<BN>::ACOL + s * KS * 32 + qq * 8);
#pragma unroll
            for (int a = 0; a < KS; ++a) tmem_st8(ta + (uint32_t)(a * 32), ops[a][0], ops[a][1]);
            tmem_wait_st();
            tc_fence_before();
          } else {
#pragma unroll
            for (int a = 0; a < KS; ++a) {
              uint8_t* arow = smem + L::OFF_A + s * L::A_BYTES + a * L::A_ATOM + r * 128;
              *reinterpret_cast<uint4*>(arow + (((2 * qq) ^ (r & 7)) << 4)) = ops[a][0];
              *reinterpret_cast<uint4*>(arow + (((2 * qq + 1) ^ (r & 7)) << 4)) = ops[a][1];
            }
            fence_proxy_async();
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&full[s]);
          if (warp == 0 && lane == 0) trace(g, it, 2);
        }
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(&emptyQ[qs]);
        }
      }
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + 4) {
    // ---------------------------------------------------------------- epilogue (4 warps)
    const int quad = warp - kEpiWarp0;
    const int r = quad * 32 + lane;
    using AT = typename std::conditional<F16, __half, __nv_bfloat16>::type;
    AT* out_act = reinterpret_cast<AT*>(g.out_act);
    float* xch = reinterpret_cast<float*>(smem + L::OFF_XCH);
    const bool atomic = g.k_splits > 1;  // split-K: partial tiles combined in a fixed order
    __shared__ int split_last_s;
    pdl_wait();
    const uint32_t rs_ep = g.mode == EPI_RS_PUSH ? *g.rs.epoch + 1 : 0u;
    int tc = 0;
    for (int u = blockIdx.x; u < tm.total; u += gridDim.x, ++tc) {
      const Tile tl = tm.decode(u);
      const int nt = tl.nt, z = tl.z;
      int gb, ge;
      grange(z, gb, ge);
      const int nacc = (ge - gb) * SPG < NI ? (ge - gb) * SPG : NI;  // issuers that wrote this tile
      const int buf = tc & 1, use = tc >> 1;
      mbar_wait(&accFull[buf], use & 1, err, 7);
      tc_fence_after();
      // All 128 epilogue threads agree on stopping (the error word only ever grows).
      asm volatile("bar.sync 2, 128;" ::: "memory");
      if (*err) break;
      const int n0 = tl.n0, t0 = tl.row0, t_end = tl.row0 + tl.rows, n = n0 + r;
      const int split_tile = nt + tm.n_tiles * (t0 / BN);  // output tile id (split-K, RS flags)
      const uint32_t acc = tmem + (uint32_t)(buf * NI * BN) + ((uint32_t)(quad * 32) << 16);
      for (int c0 = 0; c0 < BN; c0 += 32) {
        float v[32];
        tmem_ld32(acc + (uint32_t)c0, v);
        for (int m = 1; m < nacc; ++m) {
          float w[32];
          tmem_ld32(acc + (uint32_t)(m * BN + c0), w);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] += w[j];
        }
        if (g.mode == EPI_SWIGLU_Q8 && !atomic) {
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
              if (t < t_end && f < g.N / 2)
                out_act[(size_t)t * g.ld_out + f] = from_f<AT>(silu(v[j]) * up[j * 32 + lane]);
            }
          }
          asm volatile("bar.sync 2, 128;" ::: "memory");
          continue;
        }
        if (n < g.N) {
          const float bias = (g.bias && z == 0) ? g.bias[n] : 0.f;
          float* part = atomic ? g.split_ws + ((size_t)split_tile * g.k_splits + z) * BN * 128 : nullptr;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int t = t0 + c0 + j;
            if (t >= t_end) continue;
            const size_t idx = (size_t)t * g.ld_out + n;
            const float val = v[j] + bias;
            if (g.mode == EPI_MOE_COMBINE) {
              // weighted expert output of sorted row t; moe_combine sums a token's rows in slot order
              g.out_f32[idx] = g.row_w[t] * val;
            } else if (g.mode == EPI_STORE_BF16) {
              out_act[idx] = from_f<AT>(val);
            } else if (atomic) {
              part[(size_t)(c0 + j) * 128 + r] = val;
            } else if (g.mode == EPI_RS_PUSH) {
              // reduce-scatter: this rank's partial of row t goes straight into its owner's slot
              const int o = t / g.rs.chunk;
              g.rs.slots[o][((size_t)g.rs.rank * g.rs.chunk + (t - o * g.rs.chunk)) * g.N + n] = val;
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
      if (atomic) {
        // the accumulator is released; combine the splits of this tile if this split is the last
        __threadfence();
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (quad == 0 && lane == 0) split_last_s = atomicAdd(g.split_cnt + split_tile, 1) == g.k_splits - 1;
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (split_last_s) {
          __threadfence();
          const int ncol = t_end - t0;
          const float* bz = g.split_ws + (size_t)split_tile * g.k_splits * BN * 128;
          if (g.mode == EPI_SWIGLU_Q8) {
            // thread -> output feature f (rows: gate 64*(f/32) + f%32, up 32 rows later) and every
            // other column; splits summed in order, then silu(gate) * up
            const int tid = quad * 32 + lane, f = tid & 63, rg = (f >> 5) * 64 + (f & 31);
            const int fo = n0 / 2 + f;
            for (int c = tid >> 6; c < ncol && fo < g.N / 2; c += 2) {
              float sg = 0.f, su = 0.f;
              for (int zb = 0; zb < g.k_splits; zb += 4) {
                float vg[4], vu[4];
#pragma unroll
                for (int zz = 0; zz < 4; ++zz) {
                  const bool in = zb + zz < g.k_splits;
                  const float* src = bz + ((size_t)(zb + zz) * BN + c) * 128;
                  vg[zz] = in ? __ldcg(src + rg) : 0.f;
                  vu[zz] = in ? __ldcg(src + rg + 32) : 0.f;
                }
#pragma unroll
                for (int zz = 0; zz < 4; ++zz) {
                  sg += vg[zz];
                  su += vu[zz];
                }
              }
              out_act[(size_t)(t0 + c) * g.ld_out + fo] = from_f<AT>(silu(sg) * su);
            }
          } else {
            // thread (quad, lane): rows 4*lane .. 4*lane+3 of the tile, columns quad, quad+4, ...;
            // float4 loads of 4 splits of two columns are issued together, summed in split order
            const int r4 = lane * 4, n4 = n0 + r4;
            const float* base = bz + r4;
            for (int c = quad; c < ncol && n4 < g.N; c += 8) {
              float4 acc2[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
              for (int zb = 0; zb < g.k_splits; zb += 4) {
                float4 v[2][4];
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                  for (int zz = 0; zz < 4; ++zz)
                    v[h][zz] = (zb + zz < g.k_splits && c + 4 * h < ncol)
                                   ? __ldcg(reinterpret_cast<const float4*>(base + ((size_t)(zb + zz) * BN + c + 4 * h) * 128))
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                  for (int zz = 0; zz < 4; ++zz) {
                    acc2[h].x += v[h][zz].x;
                    acc2[h].y += v[h][zz].y;
                    acc2[h].z += v[h][zz].z;
                    acc2[h].w += v[h][zz].w;
                  }
              }
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                if (c + 4 * h >= ncol) break;
                float4 s4 = acc2[h];
                const int t = t0 + c + 4 * h;
                if (g.mode == EPI_RS_PUSH) {  // the summed tile goes to its owner (reduce-scatter)
                  const int ow = t / g.rs.chunk;
                  *reinterpret_cast<float4*>(g.rs.slots[ow] + ((size_t)g.rs.rank * g.rs.chunk + (t - ow * g.rs.chunk)) *
                                                                  g.N + n4) = s4;
                  continue;
                }
                float4* o = reinterpret_cast<float4*>(g.out_f32 + (size_t)t * g.ld_out + n4);
                if (g.mode == EPI_ADD_F32) {
                  const float4 prev = *o;
                  s4.x += prev.x;
                  s4.y += prev.y;
                  s4.z += prev.z;
                  s4.w += prev.w;
                }
                *o = s4;
              }
            }
          }
          if (quad == 0 && lane == 0) g.split_cnt[split_tile] = 0;
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");  // split_last_s is read before the next tile
      }
      if (g.mode == EPI_RS_PUSH && (!atomic || split_last_s)) {
        // (split-K: only the split that summed the tile pushed it)
        // every thread's stores reach the owners before the tile's flag (release at system scope)
        __threadfence_system();
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (quad == 0 && lane < g.rs.world) {
          const int o = lane;
          if (o * g.rs.chunk < t_end && (o + 1) * g.rs.chunk > t0)
            st_release_sys(g.rs.flags[o] + (size_t)g.rs.rank * g.rs.max_tiles + split_tile, rs_ep);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, Issuers<BN>::COLS);
  }
  if (threadIdx.x == 0 && err_s && g.err) atomicExch(g.err, err_s);
}

// ------------------------------------------------------------------------------------ dense dequant
// Whole weight -> row-major fp16/bf16 [N, K], one CTA per tiled chunk (128 rows x G columns): the
// chunk is staged in shared memory with 16-byte loads, then each thread expands 32-weight
// sub-blocks with the GEMM's own dequant32 and writes 64 contiguous bytes.  Used for large-T
// prefill, where dequantizing once and running a dense tensor-core GEMM beats expanding every
// weight tile inside the GEMM mainloop.
template <int WT, bool F16>
__global__ void __launch_bounds__(512) dequant_dense_kernel(const uint8_t* __restrict__ w, int N, int K,
                                                           void* __restrict__ out) {
  using F = TileFmt<WT>;
  __shared__ __align__(16) uint8_t ch[F::CHUNK];
  const int KG = K / F::G;
  const int nt = blockIdx.x / KG, kg = blockIdx.x % KG;
  const uint4* src = reinterpret_cast<const uint4*>(w + (size_t)blockIdx.x * F::CHUNK);
  for (int i = threadIdx.x; i < F::CHUNK / 16; i += blockDim.x) reinterpret_cast<uint4*>(ch)[i] = src[i];
  __syncthreads();
  constexpr int SB = F::G / 32;  // 32-weight sub-blocks per chunk row
  using AT = typename std::conditional<F16, __half, __nv_bfloat16>::type;
  AT* o = reinterpret_cast<AT*>(out);
  for (int task = threadIdx.x; task < 128 * SB; task += blockDim.x) {
    const int r = task / SB, j8 = task % SB;
    const int row = nt * 128 + r;
    if (row >= N) continue;
    uint4 v[4];
    dequant32<WT, F16>(ch, r, j8 >> 1, j8 & 1, v);
    uint4* dst = reinterpret_cast<uint4*>(o + (size_t)row * K + (size_t)kg * F::G + j8 * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) dst[i] = v[i];
  }
}

template <int WT>
static int launch_dense(const QW& w, void* out, int f16, cudaStream_t st) {
  using F = TileFmt<WT>;
  const int blocks = ((w.N + 127) / 128) * (w.K / F::G);
  cudaError_t e = f16 ? launch_pdl(dequant_dense_kernel<WT, true>, dim3(blocks), dim3(512), 0, st, w.p0, w.N, w.K, out)
                      : launch_pdl(dequant_dense_kernel<WT, false>, dim3(blocks), dim3(512), 0, st, w.p0, w.N, w.K, out);
  return e == cudaSuccess ? 0 : -20;
}

int dequant_dense(const QW& w, void* out, int out_f16, cudaStream_t st) {
  const int G = (w.type == W_Q4_K || w.type == W_Q5_K || w.type == W_Q6_K) ? 256 : 64;
  if (w.K % G) return -2;
  if ((reinterpret_cast<uintptr_t>(out) & 15) || (reinterpret_cast<uintptr_t>(w.p0) & 15)) return -3;
  switch (w.type) {
    case W_Q4_K: return launch_dense<W_Q4_K>(w, out, out_f16, st);
    case W_Q5_K: return launch_dense<W_Q5_K>(w, out, out_f16, st);
    case W_Q6_K: return launch_dense<W_Q6_K>(w, out, out_f16, st);
    case W_Q8_0: return launch_dense<W_Q8_0>(w, out, out_f16, st);
    case W_Q4_0: return launch_dense<W_Q4_0>(w, out, out_f16, st);
    case W_IQ4_NL: return launch_dense<W_IQ4_NL>(w, out, out_f16, st);
  }
  return -7;
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

static int make_act_map(CUtensorMap* m, const void* base, bool f16, int K, int T, int bn) {
  auto enc = get_encode();
  if (!enc) return -10;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)bn};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
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

int* kernel_err_word() { return device_err_word(); }

// Split-K workspace, one per device, allocated on the first split call (before any graph capture:
// the engine runs eager steps first).  The counters are left zero by the kernel.
constexpr long kSplitWsFloats = 160L * 128 * 256;  // 20 MiB
constexpr int kSplitCounters = 4096;
struct SplitWs {
  float* ws;
  int* cnt;
};

static const SplitWs* device_split_ws() {
  int dev = 0;
  cudaGetDevice(&dev);
  static std::mutex mu;
  static std::unordered_map<int, SplitWs> bufs;
  std::lock_guard<std::mutex> lk(mu);
  auto it = bufs.find(dev);
  if (it != bufs.end()) return &it->second;
  SplitWs w{nullptr, nullptr};
  if (cudaMalloc(&w.ws, kSplitWsFloats * sizeof(float)) != cudaSuccess) return nullptr;
  if (cudaMalloc(&w.cnt, kSplitCounters * sizeof(int)) != cudaSuccess || cudaMemset(w.cnt, 0, kSplitCounters * sizeof(int)) != cudaSuccess) {
    cudaFree(w.ws);
    return nullptr;
  }
  return &(bufs[dev] = w);
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

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

template <int WT, int BN, int S, int SQ, int KS, bool F16>
static int launch_gemm(const CUtensorMap& tx, const GemmDev& g, int tiles_t, cudaStream_t st) {
  using L = GemmSmem<WT, BN, S, SQ, KS>;
  static_assert(L::TOTAL + 4096 <= 232448, "shared memory budget (dynamic + static)");
  auto kern = qgemm_tc_kernel<WT, BN, S, SQ, KS, F16>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL) != cudaSuccess) return -21;
  const int n = sm_count();
  const int total = g.ng ? n : ((g.N + 127) / 128) * tiles_t * g.k_splits;  // grouped: sized on the device
  return launch_pdl(kern, dim3(total < n ? total : n), dim3(kThreads), (size_t)L::TOTAL, st, tx, g) == cudaSuccess ? 0
                                                                                                          : -20;
}

// Weight-chunk ring depth: as many chunks in flight as the shared memory left after the operand
// rings allows (capped at 8), so each SM keeps tens of KB of weight loads outstanding.
template <int WT, int BN, int S, int KS>
constexpr int chunk_slots() {
  using L = GemmSmem<WT, BN, S, 1, KS>;
  // + static shared memory of the kernel (grouped-GEMM tables, error word): 4 KB reserved
  constexpr int fixed = L::OFF_Q + L::XCH_BYTES + (2 + 2 * S + 4) * 8 + 16 + 1024 + 1024 + 4096;
  constexpr int n = (232448 - fixed) / L::Q_BYTES;
  return n > 8 ? 8 : n;
}

template <int WT, bool F16>
static int dispatch_bn(const void* x, const GemmDev& g0, cudaStream_t st) {
  using F = TileFmt<WT>;
  // K-quant chunks are 256 columns wide: small token tiles take two 64-column atoms per stage, so
  // the MMA thread issues 8 MMAs per barrier round instead of 4
  constexpr int KSW = F::G >= 128 ? 2 : 1;
  GemmDev g = g0;
  const int rows_per_tile = g.ng ? (g.T + g.ng - 1) / g.ng : g.T;  // grouped: mean rows per group
  const int bn = gemm_tile_rows(rows_per_tile);
  CUtensorMap mx;
  int rc = make_act_map(&mx, x, F16, g.K, g.T, bn);
  if (rc) return rc;
  const int tiles_t = (g.T + bn - 1) / bn;
  const int KG = g.K / F::G;
  if (g.k_splits == 0) {  // automatic split-K so that small token counts still fill the SMs
    const int tiles = ((g.N + 127) / 128) * tiles_t, n = sm_count();
    int ks = 1;
    if ((g.mode == EPI_STORE_F32 || g.mode == EPI_ADD_F32 || g.mode == EPI_RS_PUSH || g.mode == EPI_SWIGLU_Q8) &&
        g.ld_out % 4 == 0 && g.N % 4 == 0)
      // more splits only while the work units still fit one wave of CTAs
      while (ks < kMaxAutoSplits && tiles * ks * 2 <= n && KG / (ks * 2) >= 2) ks *= 2;
    g.k_splits = ks;
  }
  if (g.k_splits > KG) g.k_splits = KG;
  if (g.k_splits > kMaxAutoSplits) g.k_splits = kMaxAutoSplits;
  if (g.k_splits > 1 && (g.ld_out % 4 || g.N % 4 ||
                         (g.mode != EPI_RS_PUSH && g.mode != EPI_SWIGLU_Q8 &&
                          (reinterpret_cast<uintptr_t>(g.out_f32) & 15))))
    g.k_splits = 1;
  if (g.k_splits > 1) {
    const long tiles = (long)((g.N + 127) / 128) * tiles_t;
    // the split workspace holds kSplitWsFloats; fewer splits when a call would need more
    while (g.k_splits > 1 && (tiles * g.k_splits * bn * 128 > kSplitWsFloats || tiles > kSplitCounters)) g.k_splits /= 2;
    if (g.k_splits > 1) {
      const SplitWs* w = device_split_ws();
      if (!w) return -6;
      g.split_ws = w->ws;
      g.split_cnt = w->cnt;
    }
  }
  // TS tiles: the operand stages fill the TMEM columns left after the accumulators (256 of 512)
  constexpr int S_TS = 256 / (KSW * 32);
  // 32-row token tiles (<= 32 tokens): half the MMA width of a 64-row tile, and the TMEM the smaller
  // accumulators leave free holds 6 operand stages instead of 4
  constexpr int S32 = kGemmTS ? (512 - Issuers<32>::ACOL) / (KSW * 32) : 4;
  constexpr int S64 = kGemmTS ? S_TS : 3;
  constexpr int S128 = kGemmTS ? S_TS : 2;
  if (bn == 32) return launch_gemm<WT, 32, S32, chunk_slots<WT, 32, S32, KSW>(), KSW, F16>(mx, g, tiles_t, st);
  if (bn == 64) return launch_gemm<WT, 64, S64, chunk_slots<WT, 64, S64, KSW>(), KSW, F16>(mx, g, tiles_t, st);
  if (bn == 128) return launch_gemm<WT, 128, S128, chunk_slots<WT, 128, S128, KSW>(), KSW, F16>(mx, g, tiles_t, st);
  return launch_gemm<WT, 256, 3, chunk_slots<WT, 256, 3, 1>(), 1, F16>(mx, g, tiles_t, st);
}

template <bool F16>
static int dispatch_type(int type, const void* x, const GemmDev& g, cudaStream_t st) {
  switch (type) {
    case W_Q4_K: return dispatch_bn<W_Q4_K, F16>(x, g, st);
    case W_Q5_K: return dispatch_bn<W_Q5_K, F16>(x, g, st);
    case W_Q6_K: return dispatch_bn<W_Q6_K, F16>(x, g, st);
    case W_Q8_0: return dispatch_bn<W_Q8_0, F16>(x, g, st);
    case W_Q4_0: return dispatch_bn<W_Q4_0, F16>(x, g, st);
    case W_IQ4_NL: return dispatch_bn<W_IQ4_NL, F16>(x, g, st);
  }
  return -7;
}

static unsigned long long* g_trace = nullptr;
void gemm_set_trace(void* p) { g_trace = reinterpret_cast<unsigned long long*>(p); }

int qgemm_tc(const QW& w, const void* x, int x_is_f16, int T, const GemvEpi& ep, int k_splits, cudaStream_t st,
             const GemmGroups* grp, const SpPush* rs, const SpWait* agw) {
  if (T <= 0) return 0;
  if (ep.mode == EPI_RS_PUSH) {
    if (!rs || grp || rs->world < 1 || rs->world > kSpMaxRanks || rs->rank < 0 || rs->rank >= rs->world ||
        rs->chunk * rs->world < T || !rs->epoch)
      return -12;
    const int tiles = ((w.N + 127) / 128) * ((T + gemm_tile_rows(T) - 1) / gemm_tile_rows(T));
    if (tiles > rs->max_tiles) return -13;
    for (int q = 0; q < rs->world; ++q)
      if (reinterpret_cast<uintptr_t>(rs->slots[q]) & 15) return -12;
  }
  if (agw && (grp || !agw->flags || !agw->epoch)) return -14;
  if (grp) {
    if (grp->ng <= 0 || grp->ng > kMaxGroups || grp->grows % 128 || (long)grp->ng * grp->grows != w.N) return -8;
    if (ep.mode == EPI_MOE_COMBINE && (!grp->row_tok || !grp->row_w)) return -9;
    k_splits = 1;
  } else if (ep.mode == EPI_MOE_COMBINE) {
    return -9;
  }
  const int G = (w.type == W_Q4_K || w.type == W_Q5_K || w.type == W_Q6_K) ? 256 : 64;
  if (w.K % G) return -2;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w.p0) & 15)) return -3;
  if (ep.mode == EPI_SWIGLU_Q8 && (grp ? grp->grows : w.N) % 128) return -4;
  if (ep.mode == EPI_STORE_BF16) k_splits = 1;
  if (k_splits < 0) k_splits = 0;
  GemmDev g;
  g.N = grp ? grp->grows : w.N;
  g.goff = grp ? grp->off : nullptr;
  g.ng = grp ? grp->ng : 0;
  g.grows = grp ? grp->grows : 0;
  g.row_tok = grp ? grp->row_tok : nullptr;
  g.row_w = grp ? grp->row_w : nullptr;
  g.K = w.K;
  g.T = T;
  g.w = w.p0;
  g.mode = ep.mode;
  g.out_f32 = ep.out_f32;
  g.out_act = ep.out_bf16;
  g.bias = ep.bias;
  g.ld_out = ep.ld_out;
  g.k_splits = k_splits;
  g.split_ws = nullptr;
  g.split_cnt = nullptr;
  g.rs = rs ? *rs : SpPush{};
  g.agw = agw ? *agw : SpWait{};
  g.err = device_err_word();
  static const int exp_flags = [] {
    const char* e = getenv("BARQ_GEMM_EXP");
    return e ? atoi(e) : 0;
  }();
  g.exp = exp_flags;
  g.trace = g_trace;
  return x_is_f16 ? dispatch_type<true>(w.type, x, g, st) : dispatch_type<false>(w.type, x, g, st);
}

}  // namespace barq
