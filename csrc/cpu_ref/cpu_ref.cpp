// C++ CPU oracle (K15): ggml-spec block dequantization and an f32 matrix-vector product.
//
// Restates, from the public ggml block definitions, what the reference computes on the CPU:
// GGUF tensors dequantized to f32 at load (barq_core/src/gguf.rs:415-519 and :522-1208) and
// an f32 GEMV/GEMM (barq_core/src/blas.rs:193-305; the Metal gemv/gemm shaders of
// barq_core/src/metal_blas.rs:79-182 compute the same y = A x / C = A B).  Used by the tests as a
// second, independent oracle next to the NumPy dequantizers, and as the timed CPU baseline.
#include <torch/extension.h>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>
#include <ATen/Parallel.h>

namespace {

float f16(const uint8_t* p) {
  uint16_t h;
  std::memcpy(&h, p, 2);
  uint32_t s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023, out;
  if (e == 0) {
    if (m == 0) {
      out = s << 31;
    } else {  // subnormal
      e = 127 - 15 + 1;
      while (!(m & 1024)) { m <<= 1; --e; }
      m &= 1023;
      out = (s << 31) | (e << 23) | (m << 13);
    }
  } else if (e == 31) {
    out = (s << 31) | (255u << 23) | (m << 13);
  } else {
    out = (s << 31) | ((e - 15 + 127) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &out, 4);
  return f;
}

const int8_t kIQ4NL[16] = {-127, -104, -83, -65, -49, -35, -22, -10, 1, 13, 25, 38, 53, 69, 89, 113};

void scale_min_k4(int j, const uint8_t* q, int& d, int& m) {
  if (j < 4) {
    d = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// One block -> y (block_size floats).  Returns block size in elements, 0 if unsupported.
int dequant_block(int type, const uint8_t* b, float* y) {
  switch (type) {
    case 2: {  // Q4_0
      float d = f16(b);
      for (int j = 0; j < 16; ++j) {
        y[j] = ((b[2 + j] & 0xF) - 8) * d;
        y[j + 16] = ((b[2 + j] >> 4) - 8) * d;
      }
      return 32;
    }
    case 20: {  // IQ4_NL
      float d = f16(b);
      for (int j = 0; j < 16; ++j) {
        y[j] = kIQ4NL[b[2 + j] & 0xF] * d;
        y[j + 16] = kIQ4NL[b[2 + j] >> 4] * d;
      }
      return 32;
    }
    case 8: {  // Q8_0
      float d = f16(b);
      for (int j = 0; j < 32; ++j) y[j] = (int8_t)b[2 + j] * d;
      return 32;
    }
    case 12:    // Q4_K
    case 13: {  // Q5_K
      float d = f16(b), dmin = f16(b + 2);
      const uint8_t* sc = b + 4;
      const uint8_t* qh = b + 16;
      const uint8_t* q = type == 12 ? b + 16 : b + 48;
      int is = 0;
      uint8_t u1 = 1, u2 = 2;
      for (int j = 0; j < 256; j += 64) {
        int s, m;
        scale_min_k4(is, sc, s, m);
        float d1 = d * s, m1 = dmin * m;
        scale_min_k4(is + 1, sc, s, m);
        float d2 = d * s, m2 = dmin * m;
        for (int l = 0; l < 32; ++l) {
          int h1 = type == 13 && (qh[l] & u1) ? 16 : 0;
          int h2 = type == 13 && (qh[l] & u2) ? 16 : 0;
          y[j + l] = d1 * ((q[l] & 0xF) + h1) - m1;
          y[j + 32 + l] = d2 * ((q[l] >> 4) + h2) - m2;
        }
        q += 32;
        is += 2;
        u1 <<= 2;
        u2 <<= 2;
      }
      return 256;
    }
    case 14: {  // Q6_K
      const uint8_t* ql = b;
      const uint8_t* qh = b + 128;
      const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
      float d = f16(b + 208);
      for (int n = 0; n < 256; n += 128) {
        for (int l = 0; l < 32; ++l) {
          int is = l / 16;
          int q1 = (int8_t)((ql[l] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
          int q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
          int q3 = (int8_t)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
          int q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
          y[n + l] = d * sc[is + 0] * q1;
          y[n + l + 32] = d * sc[is + 2] * q2;
          y[n + l + 64] = d * sc[is + 4] * q3;
          y[n + l + 96] = d * sc[is + 6] * q4;
        }
        ql += 64;
        qh += 32;
        sc += 8;
      }
      return 256;
    }
  }
  return 0;
}

int type_size(int type) {
  switch (type) {
    case 2: case 20: return 18;
    case 8: return 34;
    case 12: return 144;
    case 13: return 176;
    case 14: return 210;
  }
  return 0;
}
int block_elems(int type) { return (type == 12 || type == 13 || type == 14) ? 256 : 32; }

torch::Tensor dequantize(torch::Tensor raw, int64_t type, int64_t n_elements) {
  TORCH_CHECK(raw.dtype() == torch::kUInt8 && raw.is_contiguous() && !raw.is_cuda(), "raw: contiguous CPU uint8");
  int ts = type_size((int)type), be = block_elems((int)type);
  TORCH_CHECK(ts > 0, "cpu_ref.dequantize: unsupported type ", type);
  TORCH_CHECK(n_elements % be == 0 && raw.numel() >= n_elements / be * ts, "size mismatch");
  auto out = torch::empty({n_elements}, torch::kFloat32);
  const uint8_t* src = raw.data_ptr<uint8_t>();
  float* dst = out.data_ptr<float>();
  int64_t nb = n_elements / be;
  at::parallel_for(0, nb, 256, [&](int64_t b0, int64_t b1) {
    for (int64_t i = b0; i < b1; ++i) dequant_block((int)type, src + i * ts, dst + i * be);
  });
  return out;
}

// y[b, n] = sum_k W[n, k] x[b, k] in f32 (W dequantized row by row).
torch::Tensor qgemv(torch::Tensor raw, int64_t type, int64_t N, int64_t K, torch::Tensor x) {
  TORCH_CHECK(x.dtype() == torch::kFloat32 && x.dim() == 2 && x.size(1) == K, "x: [B, K] f32");
  int ts = type_size((int)type), be = block_elems((int)type);
  TORCH_CHECK(ts > 0 && K % be == 0, "unsupported type/shape");
  TORCH_CHECK(raw.dtype() == torch::kUInt8 && raw.is_contiguous() && !raw.is_cuda(), "raw: contiguous CPU uint8");
  TORCH_CHECK(N >= 0 && raw.numel() >= N * (K / be * ts), "qgemv: raw holds fewer than N rows of K values");
  auto xc = x.contiguous();
  int64_t B = x.size(0);
  auto out = torch::zeros({B, N}, torch::kFloat32);
  const uint8_t* src = raw.data_ptr<uint8_t>();
  const float* xp = xc.data_ptr<float>();
  float* yp = out.data_ptr<float>();
  int64_t row_bytes = K / be * ts;
  at::parallel_for(0, N, 16, [&](int64_t n0, int64_t n1) {
  std::vector<float> w(K);
  for (int64_t n = n0; n < n1; ++n) {
    for (int64_t i = 0; i < K / be; ++i) dequant_block((int)type, src + n * row_bytes + i * ts, w.data() + i * be);
    for (int64_t b = 0; b < B; ++b) {
      double acc = 0;
      for (int64_t k = 0; k < K; ++k) acc += (double)w[k] * xp[b * K + k];
      yp[b * N + n] = (float)acc;
    }
  }
  });
  return out;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "barq C++ CPU oracle";
  m.def("dequantize", &dequantize);
  m.def("qgemv", &qgemv);
}
