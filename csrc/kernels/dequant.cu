// K13 embedding gather straight from quantized rows, and row dequantization to bf16.
// Element-wise ggml-spec decoding of the planar layouts described in qweight.cuh.
#include "common.cuh"
#include "launch.h"
#include "qweight.cuh"

namespace barq {

__device__ __constant__ int8_t kIQ4NL[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                             1,    13,   25,  38,  53,  69,  89,  113};

BARQ_DEV float deq_elem(const QW& w, int row, int k) {
  const int K = w.K;
  switch (w.type) {
    case W_BF16:
      return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w.p0)[(size_t)row * K + k]);
    case W_Q4_0:
    case W_IQ4_NL: {
      int blk = k >> 5, e = k & 31;
      uint8_t byte = w.p0[(size_t)row * (K / 2) + blk * 16 + (e & 15)];
      int q = e < 16 ? (byte & 15) : (byte >> 4);
      float d = h2f(w.d[(size_t)row * (K / 32) + blk]);
      return d * (float)(w.type == W_Q4_0 ? q - 8 : kIQ4NL[q]);
    }
    case W_Q8_0: {
      int8_t q = reinterpret_cast<const int8_t*>(w.p0)[(size_t)row * K + k];
      return h2f(w.d[(size_t)row * (K / 32) + (k >> 5)]) * (float)q;
    }
    case W_Q4_K:
    case W_Q5_K: {
      int b = k >> 8, e = k & 255, j = e >> 6, hiw = (e >> 5) & 1, l = e & 31;
      const uint8_t* hdr = w.p2 + ((size_t)row * (K / 256) + b) * 16;
      float d = h2f(hdr[0] | (hdr[1] << 8)), dmin = h2f(hdr[2] | (hdr[3] << 8));
      const uint8_t* s = hdr + 4;
      int is = 2 * j + hiw, sc, m;
      if (is < 4) {
        sc = s[is] & 63;
        m = s[is + 4] & 63;
      } else {
        sc = (s[is + 4] & 0xF) | ((s[is - 4] >> 6) << 4);
        m = (s[is + 4] >> 4) | ((s[is] >> 6) << 4);
      }
      uint8_t byte = w.p0[(size_t)row * (K / 2) + b * 128 + 32 * j + l];
      int q = hiw ? (byte >> 4) : (byte & 15);
      if (w.type == W_Q5_K) {
        uint8_t h = w.p1[(size_t)row * (K / 8) + b * 32 + l];
        q += ((h >> is) & 1) << 4;
      }
      return d * sc * q - dmin * m;
    }
    case W_Q6_K: {
      int b = k >> 8, e = k & 255, n = e >> 7, r = e & 127, quarter = r >> 5, l = r & 31;
      const uint8_t* ql = w.p0 + (size_t)row * (K / 2) + b * 128 + 64 * n;
      const uint8_t* qh = w.p1 + (size_t)row * (K / 4) + b * 64 + 32 * n;
      const int8_t* sc = reinterpret_cast<const int8_t*>(w.p2) + (size_t)row * (K / 16) + b * 16 + 8 * n;
      float d = h2f(w.d[(size_t)row * (K / 256) + b]);
      int lo = (quarter & 1) ? ql[l + 32] : ql[l];
      int nib = (quarter >= 2) ? (lo >> 4) : (lo & 15);
      int hb = (qh[l] >> (2 * quarter)) & 3;
      int q = (nib | (hb << 4)) - 32;
      return d * sc[(l >> 4) + 2 * quarter] * q;
    }
  }
  return 0.f;
}

__global__ void embed_kernel(QW w, const int* __restrict__ ids, float* __restrict__ out) {
  const int t = blockIdx.x;
  const int row = ids[t];
  for (int k = threadIdx.x; k < w.K; k += blockDim.x) out[(size_t)t * w.K + k] = deq_elem(w, row, k);
}

int embed_gather(const QW& table, const int* ids, int T, float* out, cudaStream_t st) {
  if (T <= 0) return 0;
  embed_kernel<<<T, 256, 0, st>>>(table, ids, out);
  return 0;
}

__global__ void dequant_rows_kernel(QW w, int r0, __nv_bfloat16* __restrict__ out) {
  const int r = blockIdx.x;
  for (int k = threadIdx.x; k < w.K; k += blockDim.x)
    out[(size_t)r * w.K + k] = __float2bfloat16(deq_elem(w, r0 + r, k));
}

int dequant_rows(const QW& w, int r0, int n, __nv_bfloat16* out, cudaStream_t st) {
  if (n <= 0) return 0;
  dequant_rows_kernel<<<n, 256, 0, st>>>(w, r0, out);
  return 0;
}

}  // namespace barq
