// Shared device helpers for the barq sm_100a kernels.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <stdint.h>
#include "qweight.cuh"

#define BARQ_DEV __device__ __forceinline__

// Diagnostic switches inside the GEMM / streaming-GEMV mainloops (skip the dequant arithmetic, skip
// the activation copy, trace stage timestamps).  Compiled out unless built with -DBARQ_DIAG=1, so
// the product kernels carry no runtime branch for them.
#ifndef BARQ_DIAG
#define BARQ_DIAG 0
#endif

namespace barq {

constexpr bool kDiag = BARQ_DIAG != 0;


BARQ_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

BARQ_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

BARQ_DEV int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

BARQ_DEV float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

BARQ_DEV int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

BARQ_DEV float silu(float x) { return x / (1.0f + __expf(-x)); }

BARQ_DEV float to_f(float v) { return v; }
BARQ_DEV float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
BARQ_DEV float to_f(__half v) { return __half2float(v); }
BARQ_DEV float to_f(__nv_fp8_e4m3 v) { return static_cast<float>(v); }

template <typename T> BARQ_DEV T from_f(float v);
template <> BARQ_DEV float from_f<float>(float v) { return v; }
template <> BARQ_DEV __nv_bfloat16 from_f<__nv_bfloat16>(float v) { return __float2bfloat16(v); }
template <> BARQ_DEV __half from_f<__half>(float v) { return __float2half(v); }
// fp8 e4m3 KV cache: round to nearest, saturating at +-448
template <> BARQ_DEV __nv_fp8_e4m3 from_f<__nv_fp8_e4m3>(float v) { return __nv_fp8_e4m3(v); }

BARQ_DEV int4 ldg16(const void* p) { return __ldg(reinterpret_cast<const int4*>(p)); }
// Streaming 16-byte load (no L1 allocation) for weights that are read exactly once per step.
BARQ_DEV int4 ldg16_stream(const void* p) {
  int4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// Activation store in the run-time activation dtype (fp16 or bf16).
BARQ_DEV void store_act(void* p, size_t i, float v, int f16) {
  if (f16)
    reinterpret_cast<__half*>(p)[i] = __float2half(v);
  else
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16(v);
}

// Quantize 32 consecutive values held one per lane into int8 with a shared scale.
// Returns the lane's int8 value; lane 0's (d, d*sum) is written by the caller.
BARQ_DEV int8_t quant_lane32(float v, float& d_out, float& s_out) {
  float amax = warp_max(fabsf(v));
  float d = amax / 127.0f;
  float id = d > 0.f ? 1.0f / d : 0.f;
  int q = __float2int_rn(v * id);
  q = max(-127, min(127, q));
  int qs = warp_sum_int(q);
  d_out = d;
  s_out = d * (float)qs;
  return (int8_t)q;
}

// Two-term version: v ~= d*q + dl*ql.  s_out is the sum of both terms over the 32 values.
BARQ_DEV void quant_lane32x2(float v, int8_t& q, int8_t& ql, float& d_out, float& dl_out, float& s_out) {
  float amax = warp_max(fabsf(v));
  float d = amax / 127.0f;
  float id = d > 0.f ? 1.0f / d : 0.f;
  int qi = max(-127, min(127, __float2int_rn(v * id)));
  // The residual (|r| <= d/2) is quantized with the fixed step d/256, so q*256 + ql is a 16-bit code
  // of v with step d/256: consumers may fold both terms into one integer dot product.
  float r = v - d * (float)qi;
  float dl = d * (1.0f / 256.0f);
  float idl = id * 256.0f;
  int qli = max(-127, min(127, __float2int_rn(r * idl)));
  int sq = warp_sum_int(qi), sql = warp_sum_int(qli);
  q = (int8_t)qi;
  ql = (int8_t)qli;
  d_out = d;
  dl_out = dl;
  s_out = d * (float)sq + dl * (float)sql;
}

// Writes lane's value of a 32-value group into an activation (single or two-term).
BARQ_DEV void act_store32(const ActOut& o, float v, size_t elem, size_t group, int lane) {
  if (o.ql) {
    int8_t q, ql;
    float d, dl, s;
    quant_lane32x2(v, q, ql, d, dl, s);
    o.q[elem] = q;
    o.ql[elem] = ql;
    if (lane == 0) {
      o.s[group] = make_float2(d, s);
      o.dl[group] = make_float2(dl, 0.f);
    }
  } else {
    float d, s;
    int8_t q = quant_lane32(v, d, s);
    o.q[elem] = q;
    if (lane == 0) o.s[group] = make_float2(d, s);
  }
}

}  // namespace barq
