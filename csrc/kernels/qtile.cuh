// Tiled quantized-weight layout shared by the GEMV (K1), GEMM (K2), embedding and dequant kernels.
//
// A weight [N, K] is cut into chunks of 128 rows x G columns (G = 256 for K-quants, 64 for the
// 32-element block types).  Chunk (nt, kg) is contiguous in memory, so the GEMM fetches it with one
// bulk copy; inside a chunk each per-block field of GGUF (quants, high bits, scales, f16 d) is a
// separate plane [128 rows][bytes per group], all 16-byte aligned:
//
//   type    G    planes (bytes per row)                        chunk bytes
//   Q4_K   256   qs 128 | hdr 16 (d, dmin, scales[12])          18432
//   Q5_K   256   qs 128 | qh 32 | hdr 16                         22528
//   Q6_K   256   ql 128 | qh 64 | sc 16 | d 2                    26880
//   Q8_0    64   qs 64  | d 4 (two f16)                           8704
//   Q4_0    64   qs 32  | d 4                                     4608
//   IQ4_NL  64   qs 32  | d 4                                     4608
//
// Planes with 32-, 64- or 128-byte rows store their 16-byte chunks XOR-swizzled by row
// (chunk c of row r at position c ^ f(r), f = r&7, (r>>1)&3, (r>>2)&1 respectively), so that eight
// consecutive rows reading the same logical chunk hit eight different shared-memory bank groups.
// Rows past N are zero.  The map from GGUF blocks is a bijection (tests re-emit the GGUF bytes).
#pragma once
#include <stdint.h>
#include "qweight.cuh"

namespace barq {

template <int WT> struct TileFmt;
template <> struct TileFmt<W_Q4_K> {
  static constexpr int G = 256, NP = 2;
  static constexpr int rb[3] = {128, 16, 0};
  static constexpr int off[3] = {0, 128 * 128, 0};
  static constexpr int CHUNK = 128 * 144;
};
template <> struct TileFmt<W_Q5_K> {
  static constexpr int G = 256, NP = 3;
  static constexpr int rb[3] = {128, 32, 16};
  static constexpr int off[3] = {0, 128 * 128, 128 * 160};
  static constexpr int CHUNK = 128 * 176;
};
template <> struct TileFmt<W_Q6_K> {
  static constexpr int G = 256, NP = 3;  // + d plane (2 B/row) after sc
  static constexpr int rb[3] = {128, 64, 16};
  static constexpr int off[3] = {0, 128 * 128, 128 * 192};
  static constexpr int D_OFF = 128 * 208;
  static constexpr int CHUNK = 128 * 210;
};
template <> struct TileFmt<W_Q8_0> {
  static constexpr int G = 64, NP = 1;
  static constexpr int rb[3] = {64, 0, 0};
  static constexpr int off[3] = {0, 0, 0};
  static constexpr int D_OFF = 128 * 64;
  static constexpr int CHUNK = 128 * 68;
};
template <> struct TileFmt<W_Q4_0> {
  static constexpr int G = 64, NP = 1;
  static constexpr int rb[3] = {32, 0, 0};
  static constexpr int off[3] = {0, 0, 0};
  static constexpr int D_OFF = 128 * 32;
  static constexpr int CHUNK = 128 * 36;
};
template <> struct TileFmt<W_IQ4_NL> : TileFmt<W_Q4_0> {};

// Physical 16-byte chunk index of logical chunk c in a row of `row_bytes` (swizzle by row).
__host__ __device__ __forceinline__ int swz(int c, int r, int row_bytes) {
  if (row_bytes == 128) return c ^ (r & 7);
  if (row_bytes == 64) return c ^ ((r >> 1) & 3);
  if (row_bytes == 32) return c ^ ((r >> 2) & 1);
  return c;
}

// Start of chunk (nt, kg).
template <int WT>
__device__ __forceinline__ const uint8_t* chunk_ptr(const QW& w, int nt, int kg) {
  const int KG = w.K / TileFmt<WT>::G;
  return w.p0 + ((size_t)nt * KG + kg) * TileFmt<WT>::CHUNK;
}

// 16-byte logical chunk c of plane P of global row `row`, group kg.
template <int WT, int P>
__device__ __forceinline__ const uint8_t* plane_chunk(const QW& w, int row, int kg, int c) {
  using F = TileFmt<WT>;
  constexpr int RB = F::rb[P], OFF = F::off[P];
  const int r = row & 127;
  return chunk_ptr<WT>(w, row >> 7, kg) + OFF + r * RB + 16 * swz(c, r, RB);
}

// Same inside a chunk already staged in shared memory (row r = 0..127).
template <int WT, int P>
__device__ __forceinline__ const uint8_t* staged_chunk(const uint8_t* chunk, int r, int c) {
  using F = TileFmt<WT>;
  constexpr int RB = F::rb[P], OFF = F::off[P];
  return chunk + OFF + r * RB + 16 * swz(c, r, RB);
}

}  // namespace barq
