// Split-KV paged decode attention that allocates nothing: its scratch lives in a fixed,
// file-scope device array instead of memory the caller or this library allocates.
//
// This entry point has no counterpart in the reference (whose attention runs on the host).
//
// Who needs it: callers that cannot call cudaMalloc (or any allocating routine, torch's caching
// allocator included) on the path that runs attention -- for example a host process whose device
// memory is owned by another allocator or plugin host that forbids allocation from inside the
// operator, or a latency-critical loop that cannot afford cudaMalloc's implicit device-wide
// synchronization and its failure mode once the memory is already reserved elsewhere.  They
// still pass every input and output buffer; only the split-KV scratch is provided here.
//
// Limits and behaviour:
//   * Scratch is BARQ_DECODE_STATIC_SCRATCH_BYTES (8 MiB) per GPU, held by every GPU that loads
//     this library until the process exits.  A call needs
//     4 * (B*H*splits*D + B*H*splits*2) bytes plus up to 256 bytes of alignment; larger requests
//     are rejected with BARQ_STATIC_E_SCRATCH and nothing is launched.
//   * Set-up: the first call on each device (with that device current) resolves the array's device
//     address with cudaGetSymbolAddress and caches it.  Make that first call before any stream
//     capture begins.
//   * All calls on a device share the one array and it keeps the last call's contents.  Nothing in
//     it has to start at zero: the split kernel writes every partial result that the merge reads.
//     Calls whose kernels overlap on the GPU (different streams without ordering between them) race
//     on the array and produce wrong results; order them on one stream or with events.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BARQ_DECODE_STATIC_SCRATCH_BYTES (8u * 1024u * 1024u)

#define BARQ_STATIC_OK 0
#define BARQ_STATIC_E_SCRATCH (-101)  // the shape needs more scratch than the static array holds
#define BARQ_STATIC_E_SETUP (-102)    // cudaGetDevice / cudaGetSymbolAddress failed: see barq_static_last_cuda_error
#define BARQ_STATIC_E_ARGS (-103)     // null pointer, non-positive size or unsupported shape
#define BARQ_STATIC_E_LAUNCH (-104)   // a kernel launch failed: see barq_static_last_cuda_error

// q: bf16 [B, H, D]; kcache / vcache: fp16 (cache_is_bf16 = 0) or bf16 [num_blocks, Hkv, block_size, D];
// block_tables: int32 [B, max_blocks]; seq_lens: int32 [B] (tokens in the cache, current one
// included); out: [B, H*D] fp16 (out_f16 = 1) or bf16.  block_size must be 16, D 64 or 128,
// 1 <= splits <= 64, H a multiple of Hkv with H / Hkv in {1, 2, 4, 8} (other shapes return
// BARQ_STATIC_E_ARGS before anything is launched).  window > 0 limits attention to the last
// `window` tokens.
// stream: a cudaStream_t (0 = legacy default stream).  Returns BARQ_STATIC_OK or a negative code.
__attribute__((visibility("default"))) int barq_decode_attention_static(
    const void* q, const void* kcache, const void* vcache, int cache_is_bf16, const int* block_tables, int max_blocks,
    const int* seq_lens, int B, int H, int Hkv, int D, int block_size, float scale, int window, int splits, void* out,
    int out_f16, void* stream);

// Bytes of static scratch a call with this shape needs (alignment padding included).
__attribute__((visibility("default"))) unsigned long long barq_decode_attention_static_need(int B, int H, int D,
                                                                                            int splits);

// The CUDA error behind the calling thread's last BARQ_STATIC_E_SETUP or BARQ_STATIC_E_LAUNCH
// (cudaSuccess when its last call succeeded), as a cudaError_t value.
__attribute__((visibility("default"))) int barq_static_last_cuda_error(void);

// A one-line description of a return code of barq_decode_attention_static.
__attribute__((visibility("default"))) const char* barq_static_strerror(int code);

#ifdef __cplusplus
}
#endif
