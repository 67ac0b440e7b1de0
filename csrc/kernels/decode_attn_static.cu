// Decode attention with file-scope static scratch: see decode_attn_static.h for who needs it, the
// size limit and the sharing rules.  The kernels are the library's split-KV decode kernels
// (attn_decode.cu), launched through the same launcher; only where the scratch lives differs.
#include "decode_attn_static.h"

#include <atomic>
#include <mutex>

#include "launch.h"

namespace {

constexpr unsigned kScratchFloats = BARQ_DECODE_STATIC_SCRATCH_BYTES / sizeof(float);
constexpr int kMaxDevices = 64;

// The scratch itself.  In host code this name is only a handle for cudaGetSymbolAddress, never a
// device address.
__device__ __align__(256) float g_decode_scratch[kScratchFloats];

std::atomic<float*> g_dev_ptr[kMaxDevices];  // device address of g_decode_scratch, per device
std::mutex g_setup_mu;
thread_local cudaError_t g_last_cuda_error = cudaSuccess;

// Set-up, once per device, with that device current.
float* scratch_for_current_device(int* code) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    g_last_cuda_error = e;
    *code = BARQ_STATIC_E_SETUP;
    return nullptr;
  }
  float* p = g_dev_ptr[dev].load(std::memory_order_acquire);
  if (p) return p;
  std::lock_guard<std::mutex> lk(g_setup_mu);
  p = g_dev_ptr[dev].load(std::memory_order_relaxed);
  if (p) return p;
  void* addr = nullptr;
  e = cudaGetSymbolAddress(&addr, g_decode_scratch);
  if (e != cudaSuccess || addr == nullptr) {
    g_last_cuda_error = e;
    *code = BARQ_STATIC_E_SETUP;
    return nullptr;
  }
  p = static_cast<float*>(addr);
  g_dev_ptr[dev].store(p, std::memory_order_release);
  return p;
}

unsigned long long acc_floats(int B, int H, int D, int splits) {
  return (unsigned long long)B * H * splits * D;
}

}  // namespace

extern "C" unsigned long long barq_decode_attention_static_need(int B, int H, int D, int splits) {
  if (B <= 0 || H <= 0 || D <= 0 || splits <= 0) return 0;
  // part_acc, then part_ml (float2) starting on a 256-byte boundary
  const unsigned long long acc = acc_floats(B, H, D, splits);
  const unsigned long long ml_off = (acc + 63) / 64 * 64;
  return (ml_off + 2ull * B * H * splits) * sizeof(float);
}

extern "C" int barq_decode_attention_static(const void* q, const void* kcache, const void* vcache, int cache_is_bf16,
                                            const int* block_tables, int max_blocks, const int* seq_lens, int B,
                                            int H, int Hkv, int D, int block_size, float scale, int window,
                                            int splits, void* out, int out_f16, void* stream) {
  g_last_cuda_error = cudaSuccess;
  if (!q || !kcache || !vcache || !block_tables || !seq_lens || !out || B <= 0 || H <= 0 || Hkv <= 0 || D <= 0 ||
      splits <= 0 || max_blocks <= 0)
    return BARQ_STATIC_E_ARGS;
  // the launcher's own limits, checked here so that an unsupported shape is an argument error
  const int G = H % Hkv == 0 ? H / Hkv : 0;
  if (block_size != 16 || (D != 64 && D != 128) || splits > 64 || (G != 1 && G != 2 && G != 4 && G != 8))
    return BARQ_STATIC_E_ARGS;
  if (barq_decode_attention_static_need(B, H, D, splits) > BARQ_DECODE_STATIC_SCRATCH_BYTES)
    return BARQ_STATIC_E_SCRATCH;
  int code = BARQ_STATIC_OK;
  float* base = scratch_for_current_device(&code);
  if (!base) return code;

  barq::DecodeAttnArgs a;
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.kcache = kcache;
  a.vcache = vcache;
  a.cache_type = cache_is_bf16 ? barq::kCacheBF16 : barq::kCacheF16;
  a.block_tables = block_tables;
  a.max_blocks = max_blocks;
  a.seq_lens = seq_lens;
  a.B = B;
  a.H = H;
  a.Hkv = Hkv;
  a.D = D;
  a.block_size = block_size;
  a.scale = scale;
  a.window = window;
  a.splits = splits;
  const unsigned long long acc = acc_floats(B, H, D, splits);
  a.part_acc = base;
  a.part_ml = reinterpret_cast<float2*>(base + (acc + 63) / 64 * 64);
  a.out = out;
  a.out_f16 = out_f16;
  a.out_q = barq::ActOut{};  // no int8 copy of the output on this entry point
  // Each launch's own return code decides (the launcher checks them): a pending error that earlier,
  // unrelated work left on this thread is not reported as this call's failure.
  if (barq::decode_attention(a, static_cast<cudaStream_t>(stream)) != 0) {
    g_last_cuda_error = cudaGetLastError();
    return BARQ_STATIC_E_LAUNCH;
  }
  return BARQ_STATIC_OK;
}

extern "C" int barq_static_last_cuda_error(void) { return (int)g_last_cuda_error; }

extern "C" const char* barq_static_strerror(int code) {
  switch (code) {
    case BARQ_STATIC_OK: return "ok";
    case BARQ_STATIC_E_SCRATCH:
      return "decode attention: the shape needs more scratch than the 8 MiB static array "
             "(4*(B*H*splits*D + 2*B*H*splits) bytes); use fewer splits or a smaller batch";
    case BARQ_STATIC_E_SETUP:
      return "decode attention: cudaGetSymbolAddress of the static scratch failed (barq_static_last_cuda_error)";
    case BARQ_STATIC_E_ARGS:
      return "decode attention: null pointer, non-positive size or unsupported shape (block_size 16, D 64 or 128, "
             "splits 1..64, H / Hkv in {1, 2, 4, 8})";
    case BARQ_STATIC_E_LAUNCH: return "decode attention: a kernel launch failed (barq_static_last_cuda_error)";
  }
  return "unknown code";
}
