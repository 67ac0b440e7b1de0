// Device-side view of a quantized weight in the planar ("split-plane") layout.
//
// A GGUF tensor is a row-major sequence of ggml blocks whose sizes (18, 34, 144, 176, 210 bytes)
// are not multiples of 16, so rows of Q4_0/Q8_0/Q6_K blocks are not 16-byte aligned.  At load
// time every weight is split, block by block and without changing a bit, into up to four planes:
//
//   type     p0 (quants)        p1 (high bits)   p2 (per-block header)        d (f16 per block)
//   Q4_0     qs  [N, K/2]       -                -                            d  [N, K/32]
//   IQ4_NL   qs  [N, K/2]       -                -                            d  [N, K/32]
//   Q8_0     qs  [N, K]  (i8)   -                -                            d  [N, K/32]
//   Q4_K     qs  [N, K/2]       -                hdr [N, K/256, 16] (d,dmin,scales[12])
//   Q5_K     qs  [N, K/2]       qh [N, K/8]      hdr [N, K/256, 16]
//   Q6_K     ql  [N, K/2]       qh [N, K/4]      sc  [N, K/16] (i8)           d  [N, K/256]
//   BF16     w   [N, K]  (bf16)
//
// The map is a bijection (the Python side re-emits the GGUF blocks from the planes in tests) and
// every plane row starts on a 16-byte boundary when K is a multiple of 256 (32 for Q4_0/Q8_0/IQ4_NL),
// which is what both the vector loads of the GEMV kernels and the TMA boxes of the tcgen05 GEMM need.
#pragma once
#include <stdint.h>
#include <vector_types.h>

namespace barq {

enum WType : int {
  W_BF16 = 0,
  W_Q4_0 = 2,
  W_Q8_0 = 8,
  W_Q4_K = 12,
  W_Q5_K = 13,
  W_Q6_K = 14,
  W_IQ4_NL = 20,
};

// Activation in the "q8" layout consumed by the dp4a GEMV kernels: per token row of K values,
// int8 qs[K] and one float2 (scale d, d * sum(qs)) per 32 values.
// Optional second term (ql, dl): the int8 residual x - d*q quantized with its own scale, so that
// x ~= d*q + dl*ql to ~16 bits; s.y then holds the sum of both terms.
struct ActQ8 {
  const int8_t* q;   // [B, K]
  const float2* s;   // [B, K/32]
  const int8_t* ql;  // [B, K] or null
  const float2* dl;  // [B, K/32] (scale, 0) or null
};

// Output side of an activation producer (q / s required when used, ql / dl optional).
struct ActOut {
  int8_t* q;
  float2* s;
  int8_t* ql;
  float2* dl;
};

struct QW {
  const uint8_t* p0;
  const uint8_t* p1;
  const uint8_t* p2;
  const uint16_t* d;
  int N;
  int K;
  int type;
};

}  // namespace barq
