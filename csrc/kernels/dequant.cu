// K13 embedding gather straight from quantized rows, and row dequantization to bf16.
// Element-wise ggml-spec decoding of the tiled device layout described in qtile.cuh.
#include "common.cuh"
#include "pdl.cuh"
#include "launch.h"
#include "qweight.cuh"
#include "qtile.cuh"

namespace barq {

__device__ __constant__ int8_t kIQ4NL[16] = {-127, -104, -83, -65, -49, -35, -22, -10,
                                             1,    13,   25,  38,  53,  69,  89,  113};

// Byte `i` of plane P of (row, group kg), honouring the chunk swizzle.
template <int WT, int P>
BARQ_DEV uint8_t pbyte(const QW& w, int row, int kg, int i) {
  return plane_chunk<WT, P>(w, row, kg, i >> 4)[i & 15];
}
template <int WT>
BARQ_DEV float dplane(const QW& w, int row, int kg, int idx) {
  const uint8_t* p = chunk_ptr<WT>(w, row >> 7, kg) + TileFmt<WT>::D_OFF;
  return h2f(reinterpret_cast<const uint16_t*>(p)[(row & 127) * (TileFmt<WT>::G == 256 ? 1 : 2) + idx]);
}

BARQ_DEV float deq_elem(const QW& w, int row, int k) {
  const int K = w.K;
  switch (w.type) {
    case W_BF16:
      return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(w.p0)[(size_t)row * K + k]);
    case W_Q4_0:
    case W_IQ4_NL: {
      const int kg = k >> 6, e = k & 63, bi = e >> 5, l = e & 31;
      const uint8_t byte = w.type == W_Q4_0 ? pbyte<W_Q4_0, 0>(w, row, kg, 16 * bi + (l & 15))
                                            : pbyte<W_IQ4_NL, 0>(w, row, kg, 16 * bi + (l & 15));
      const int q = l < 16 ? (byte & 15) : (byte >> 4);
      const float d = dplane<W_Q4_0>(w, row, kg, bi);
      return d * (float)(w.type == W_Q4_0 ? q - 8 : kIQ4NL[q]);
    }
    case W_Q8_0: {
      const int kg = k >> 6, e = k & 63;
      const int8_t q = (int8_t)pbyte<W_Q8_0, 0>(w, row, kg, e);
      return dplane<W_Q8_0>(w, row, kg, e >> 5) * (float)q;
    }
    case W_Q4_K:
    case W_Q5_K: {
      const int kg = k >> 8, e = k & 255, j = e >> 6, hiw = (e >> 5) & 1, l = e & 31;
      const bool five = w.type == W_Q5_K;
      const uint8_t* hdr = five ? plane_chunk<W_Q5_K, 2>(w, row, kg, 0) : plane_chunk<W_Q4_K, 1>(w, row, kg, 0);
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
      const uint8_t byte = five ? pbyte<W_Q5_K, 0>(w, row, kg, 32 * j + l) : pbyte<W_Q4_K, 0>(w, row, kg, 32 * j + l);
      int q = hiw ? (byte >> 4) : (byte & 15);
      if (five) q += ((pbyte<W_Q5_K, 1>(w, row, kg, l) >> is) & 1) << 4;
      return d * sc * q - dmin * m;
    }
    case W_Q6_K: {
      const int kg = k >> 8, e = k & 255, n = e >> 7, r = e & 127, quarter = r >> 5, l = r & 31;
      const int lo = pbyte<W_Q6_K, 0>(w, row, kg, 64 * n + ((quarter & 1) ? 32 : 0) + l);
      const int nib = (quarter >= 2) ? (lo >> 4) : (lo & 15);
      const int hb = (pbyte<W_Q6_K, 1>(w, row, kg, 32 * n + l) >> (2 * quarter)) & 3;
      const int q = (nib | (hb << 4)) - 32;
      const int8_t sc = (int8_t)pbyte<W_Q6_K, 2>(w, row, kg, 8 * n + 2 * quarter + (l >> 4));
      return dplane<W_Q6_K>(w, row, kg, 0) * sc * q;
    }
  }
  return 0.f;
}

// A token id outside [0, vocab) is recorded in the device error word (0xB00) and its row reads as
// zeros: the gather never reads outside the table.
__global__ void embed_kernel(QW w, const int* __restrict__ ids, float* __restrict__ out, int* err) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int row = ids[t];
  const bool ok = row >= 0 && row < w.N;
  if (!ok && threadIdx.x == 0 && err) atomicExch(err, 0xB00);
  for (int k = threadIdx.x; k < w.K; k += blockDim.x) out[(size_t)t * w.K + k] = ok ? deq_elem(w, row, k) : 0.f;
}

int embed_gather(const QW& table, const int* ids, int T, float* out, cudaStream_t st) {
  if (T <= 0) return 0;
  return launch_pdl(embed_kernel, dim3(T), dim3(256), 0, st, table, ids, out, kernel_err_word()) == cudaSuccess
             ? 0
             : -20;
}

__global__ void dequant_rows_kernel(QW w, int r0, __nv_bfloat16* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  const int r = blockIdx.x;
  for (int k = threadIdx.x; k < w.K; k += blockDim.x)
    out[(size_t)r * w.K + k] = __float2bfloat16(deq_elem(w, r0 + r, k));
}

int dequant_rows(const QW& w, int r0, int n, __nv_bfloat16* out, cudaStream_t st) {
  if (n <= 0) return 0;
  return launch_pdl(dequant_rows_kernel, dim3(n), dim3(256), 0, st, w, r0, out) == cudaSuccess ? 0 : -20;
}

}  // namespace barq
