// Device-side view of a quantized weight.  Kernels read the tiled layout described in qtile.cuh
// (p0 = tiled chunk buffer); dense bf16 weights are plain [N, K] rows in p0.  p1/p2/d are unused by
// the tiled kernels.
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
