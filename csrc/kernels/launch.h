// Host-side launch API of the barq sm_100a kernels (plain C++ types, no torch headers), so each
// .cu file compiles quickly and the torch binding layer stays in one translation unit.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include "qweight.cuh"

namespace barq {

// KV cache element types
constexpr int kCacheF16 = 0, kCacheBF16 = 1, kCacheFP8 = 2;

enum EpiMode : int {
  EPI_STORE_F32 = 0,
  EPI_ADD_F32 = 1,
  EPI_STORE_BF16 = 2,
  EPI_SWIGLU_Q8 = 3,
  EPI_MOE_COMBINE = 4,
  EPI_AR_PUSH = 5,  // streaming GEMV only: tensor-parallel all-reduce fused into the epilogue (ArPush)
  EPI_RS_PUSH = 6,  // tcgen05 GEMM only: reduce-scatter fused into the epilogue (SpPush)
};

struct GemvEpi {
  int mode;
  float* out_f32;
  __nv_bfloat16* out_bf16;
  ActOut out_q;
  const float* bias;
  int ld_out;
};

// K1 quantized GEMV, B <= 8 tokens.  xb/ldxb are only read for bf16 weights.
int qgemv(const QW& w, const ActQ8& x, const __nv_bfloat16* xb, int ldxb, int B, const GemvEpi& ep,
          cudaStream_t st);

// K2 tcgen05 quantized GEMM: out[t, n] (+)= x[t, :] . W[n, :], x bf16 [T, K] (row pitch K).
// Modes as GemvEpi (EPI_SWIGLU_Q8 here writes bf16 silu(g)*u to out_bf16).  k_splits: 1 = none,
// 0 = automatic (f32 modes only; the last split of a tile sums the splits in order).
// x is fp16 (x_is_f16) or bf16; EPI_STORE_BF16 / EPI_SWIGLU_Q8 outputs use the same type as x.
// ---- Sequence-parallel tensor parallelism (tp_fused.cu, the EPI_RS_PUSH / AG-wait modes of the GEMM)
// T token rows are split over W ranks in contiguous chunks of `chunk` = ceil(T / W) rows; rank r owns
// rows [r * chunk, min(T, (r + 1) * chunk)) of the residual stream.
constexpr int kSpMaxRanks = 8;
// Token-tile height of the non-grouped tcgen05 GEMM for T rows (the RS flags are per GEMM tile).
inline int gemm_tile_rows(int T) { return T <= 32 ? 32 : T <= 64 ? 64 : (T <= 128 ? 128 : 256); }

// Row-parallel GEMM -> reduce-scatter: every finished output tile is stored (plain f32 stores over
// NVLink) into the owner rank's receive slots [src rank][chunk][N], then flagged there with the
// call's epoch (flags [src rank][max_tiles], tile id = n tile + n_tiles * token tile).
struct SpPush {
  float* slots[kSpMaxRanks];
  uint32_t* flags[kSpMaxRanks];
  const uint32_t* epoch;  // this site's call counter (advanced by sp_reduce_norm_ag)
  int rank, world, chunk, max_tiles;
};

// All-gather consumer: before loading token tile rows [t0, t1) of its activation, the GEMM waits for
// flags[t0 .. t1) (one per row, written by the owner's sp_reduce_norm_ag) to reach *epoch.
struct SpWait {
  const uint32_t* flags;
  const uint32_t* epoch;
  unsigned long long wait_ns;
};

// Owner side: x[own rows] += sum over source ranks (rank order) of the received slots (+ bias), then
// RMSNorm(x) * norm_w -> bf16 rows pushed into every rank's gather buffer ag[q][row] with a flag per
// row.  n_src = 0: no reduce (the first layer's norm after the embedding).
struct SpReduceArgs {
  const float* slots;          // this rank's receive slots [W][chunk][H]
  const uint32_t* rs_flags;    // [W][max_tiles]
  int n_src, max_tiles, gemm_bn, n_tiles;
  const float* bias;           // [H] or null (row-parallel bias, added once)
  float* x;                    // residual rows of this rank [rows][H] (row pitch H)
  int T, W, rank, chunk, H;
  const float* norm_w;
  float eps;
  int out_f16;                 // gather buffers hold fp16 (1) or bf16 (0) rows
  int self_only;               // 1: write only this rank's gather buffer (the rows feed a local op)
  void* ag[kSpMaxRanks];       // every rank's gather buffer [T][H]
  uint32_t* ag_flags[kSpMaxRanks];  // every rank's row flags [T]
  uint32_t* epoch;             // this site's call counter: ep = *epoch + 1, advanced by the last CTA
  int* done;                   // CTA arrival counter (zero between calls)
  int* err;
  unsigned long long wait_ns;
};
int sp_reduce_norm_ag(const SpReduceArgs& a, cudaStream_t st);
// Wait (on the device) until the gather flags of rows [0, T) reach *epoch: orders later plain kernels
// (torch ops) after the remote pushes.
int sp_ag_wait(const uint32_t* flags, const uint32_t* epoch, int T, int* err, unsigned long long wait_ns,
               cudaStream_t st);

// One-shot all-reduce + residual add over peer memory (allreduce.cu).
constexpr int kArMaxRanks = 8;
constexpr int kArMaxBlocks = 64;
struct ArArgs {
  float* x;                          // local residual [n], x += sum of partials
  const float* bufs[kArMaxRanks];    // every rank's partial buffer (peer pointers; bufs[rank] local)
  uint32_t* flags[kArMaxRanks];      // every rank's flag area [kArMaxBlocks][kArMaxRanks] (peer pointers)
  uint32_t* epoch;                   // local [kArMaxBlocks] epoch counters (zero-initialized)
  int* err;                          // error word (0x300 | peer on a barrier timeout)
  int rank, world, n, blocks;
  unsigned long long wait_ns;        // barrier wait limit
  int skip_signal;                   // fault injection: do not signal the peers (their waits run out)
  float* mc = nullptr;               // multicast address of this call's partial buffer (NVLS form), or null
};
int allreduce_add(const ArArgs& a, cudaStream_t st);

// DeepSeek-V2 MLA (mla.cu).  Latent cache rows: [c (512) | k_pe (64)], 16 tokens per page.
struct MlaKvArgs {
  const float* kv_a;    // [T, 576] kv_a_mqa projection
  const float* norm_w;  // [512] attn_kv_a_norm
  float eps;
  const float* cos;     // [max_pos, 32] (YaRN mscale folded in)
  const float* sin;
  int neox;
  const int* pos;       // [T]
  const int64_t* slots; // [T] cache slot = block * 16 + offset
  void* cache;          // [blocks, 16, 576] fp16 / bf16
  float* q;             // [T, H, qdim] f32; rope part rotated in place
  int T, H, qdim, rope_off;
};
int mla_kv_write(const MlaKvArgs& a, int cache_is_bf16, cudaStream_t st);

struct MlaAttnArgs {
  const float* q_lat;  // [rows, H, 512] absorbed queries
  const float* q_pe;   // rows of [H, q_pe_stride]: rotated rope part at offset 0 (pointer pre-offset)
  int q_pe_stride;     // floats between consecutive heads' q_pe (qdim)
  const void* cache;
  const int* block_tables;  // [S, max_blocks]
  int max_blocks;
  const int* row_seq;  // [rows] sequence of each query row
  const int* row_len;  // [rows] visible cache tokens (causal: position + 1)
  int rows, H, splits;
  float scale;
  float* part_acc;     // scratch [rows, splits, H, 512]
  float2* part_ml;     // scratch [rows, splits, H]
  float* o_lat;        // [rows, H, 512]
  int* err = nullptr;  // error word of the tensor-core kernel (0xA00: block-table entry out of range)
  int num_blocks = 0;  // cache pages, for that check (0: unchecked)
};
size_t mla_attn_scratch_floats(int rows, int splits);
// impl 0: CUDA-core kernel; 1: tensor-core kernel (mma.m16n8k16 over a copy-warp page ring)
int mla_attention(const MlaAttnArgs& a, int cache_is_bf16, cudaStream_t st, int impl = 0);

// MoE routing + dispatch (moe.cu).  logits f32 [T, E] -> ids/weights [T, k]; rows of x (fp16/bf16
// [T, H]) are copied into xs [T*k, H] sorted by expert, off [E+1] holds each expert's row range, and
// row_tok / row_w the source token and gate weight of each row.  counts [E] must be zero before the
// first call (the kernels leave them zero); cursor [E] is scratch.
struct MoeRouteArgs {
  const float* logits;
  int T, E, k, H;
  int sigmoid, renorm, n_group, topk_group;
  float ser_threshold, scale;
  int* ids;
  float* weights;
  int* counts;
  int* cursor;
  int* off;
  int* row_tok;
  float* row_w;
  int* tok_row;  // [T * k] sorted row of (token, slot), -1 when SER dropped the slot
};
int moe_route(const MoeRouteArgs& a, const void* x, int x_is_f16, void* xs, cudaStream_t st);
// Router logits out[T, E] (f32) = x[T, H] (fp16 / bf16, row pitch ldx) . W[E, H]^T (f32), H % 4 == 0.
int moe_router_logits(const void* x, int x_is_f16, int ldx, const float* w, float* out, int T, int E, int H,
                      cudaStream_t st);

// ---- Expert parallelism: all-to-all dispatch / combine over NVLink peer memory (moe.cu).
// Each rank routes its own token rows (sequence-parallel residual), sends every (token, slot) row to
// the rank that holds the expert, and later gathers the expert outputs back.  Receive layout on
// rank q: its E_local experts in order, each expert's rows grouped by source rank in rank order.
struct EpArgs {
  int rank, W, E, E_local, k, H, rows;  // rows: token rows of this rank
  const int* ids;          // [rows, k] expert of each slot (routing of this rank's rows)
  const float* weights;    // [rows, k] gate weight (0: slot dropped by SER)
  int* counts;             // [E] rows of this rank per expert (from the routing kernel; cleared here)
  int* cursor;             // [E] zeroed claim counters (left zero)
  int* cnt_all[kSpMaxRanks];        // every rank's count matrix [W][E]
  uint32_t* cnt_flags[kSpMaxRanks];  // every rank's count flags [W]
  const void* x;           // this rank's normalized rows [rows, H] (fp16 / bf16)
  void* recv_x[kSpMaxRanks];          // every rank's receive rows [cap, H]
  uint32_t* disp_flags[kSpMaxRanks];  // every rank's dispatch flags [W]
  int2* disp_pos;          // [rows, k] (dest rank, receive row) of each slot; dest -1: dropped
  int* recv_off;           // [E_local + 1] receive-row offsets of this rank's experts (written here)
  const float* ys[kSpMaxRanks];       // every rank's expert outputs [cap, H] f32
  uint32_t* ys_flags[kSpMaxRanks];    // every rank's "outputs ready" flags [W]
  float* out;              // this rank's residual rows [rows, H] (combine adds into it)
  uint32_t* epoch;         // EP call counter (advanced by the combine's last CTA)
  int* done;               // [2] CTA arrival counters (zero between calls)
  int cap;                 // receive rows per rank
  int* err;
  unsigned long long wait_ns;
};
// route counts of this rank -> every rank's count matrix; then dispatch rows; grouped GEMMs on the
// receive rows run in between; then signal + combine.
int ep_dispatch(const EpArgs& a, int x_is_f16, cudaStream_t st);
int ep_combine(const EpArgs& a, cudaStream_t st);

// K7 combine: x[t, :] += sum over slots j (in slot order) of ys[tok_row[t*k+j], :], counting only
// rows inside [*lo, *hi) (this rank's experts; device pointers into the routing offsets).
struct MoeCombineArgs {
  const float* ys;
  int ld_ys;
  const int* tok_row;
  const int* lo;
  const int* hi;
  int T, k, H;
  float* x;
  int ld_x;
};
int moe_combine(const MoeCombineArgs& a, cudaStream_t st);

// Grouped (MoE expert) GEMM: the weight is ng stacked groups of grows rows; activation rows sorted by
// group with device offsets off[ng+1]; EPI_MOE_COMBINE stores row_w[r] * y[r, :] into out row r (the
// sorted row), and moe_combine then sums each token's rows in a fixed order.
struct GemmGroups {
  const int* off;
  int ng, grows;
  const int* row_tok;
  const float* row_w;
};
int qgemm_tc(const QW& w, const void* x, int x_is_f16, int T, const GemvEpi& ep, int k_splits, cudaStream_t st,
             const GemmGroups* grp = nullptr, const SpPush* rs = nullptr, const SpWait* agw = nullptr);
// Whole quantized weight (tiled layout) -> row-major fp16 (out_f16) or bf16 [N, K].
int dequant_dense(const QW& w, void* out, int out_f16, cudaStream_t st);
int gemm_error_word(int* host_out);
int* kernel_err_word();  // device error word shared by the bounded-wait kernels (per device)
// f32 workspace floats the streaming GEMV needs for N output rows (one 8 x 128 slot per CTA piece).
inline long qgemv_stream_ws_floats(int N) { return ((long)(N + 127) / 128 + 256) * 8 * 128; }
// Streaming decode GEMV (1..8 tokens): persistent, bulk-copy fed, stream-K over weight chunks.
// ws_acc: f32 [8, N] and ws_cnt: int [N/128], both zero before the first call; the kernel leaves
// them zero.  Calls sharing a workspace must not overlap on the GPU.  err: bounded-wait error word.
// norm_h (optional, f32 [B, K], K <= 4096, B <= 2): the activation is computed in the kernel as
// int8(rmsnorm(norm_h) * norm_w) (two-term if norm_x2) instead of being read from x.
// Fused GEMV + all-reduce (EPI_AR_PUSH): the CTA that finishes an output tile stores it into every
// peer's receive buffer (slot = this rank) over NVLink as (epoch, value) 64-bit words, then waits
// (bounded) for the peers' words of the same tile and adds the world's sum into the residual x.
struct ArPush {
  uint64_t* const* dst;          // device table: receive buffer j of every rank, [world][B][N] words
                                 // (epoch << 32 | f32 bits); a table in memory, not a parameter
                                 // array, so that indexing it by rank needs no local-memory copy
  uint32_t* epoch;               // this rank's epoch of buffer j (device)
  int* done;                     // this rank's CTA-exit counter for buffer j (zero between calls)
  float* x;                      // residual stream [B, ld_x]
  int ld_x, rank, world, skip_signal;
  unsigned long long wait_ns;
};
int qgemv_stream(const QW& w, const ActQ8& x, int B, const GemvEpi& ep, float* ws_acc, int* ws_cnt, int* err,
                 const float* norm_h, const float* norm_w, float norm_eps, int norm_x2, cudaStream_t st,
                 const ArPush* ar = nullptr);
void gemm_set_trace(void* p);  // diagnostics (BARQ_GEMM_EXP bit 1): [256 stages][8] u64 stamps of CTA 0
int gemm_clear_error_word();

// Fused (residual add +) RMSNorm.  x: f32 [T, H] residual stream (updated in place when `add`
// is given: x += add).  Outputs any of bf16 [T, H] and int8 q8 [T, H] + scales [T, H/32].
int rmsnorm(float* x, const float* add, const float* w, float eps, int T, int H, void* out_act, int out_f16,
            ActOut out_q, cudaStream_t st);

// Quantize bf16 or f32 rows to the q8 activation layout (H % 32 == 0).
int quantize_q8(const void* x, int x_is_bf16, int T, int H, int ldx, ActOut out_q, cudaStream_t st);

// h = silu(g) * u with g = in[t, i], u = in[t, F + i] (f32 or bf16 input) -> bf16 and/or q8.
int swiglu(const void* in, int in_is_bf16, int T, int F, int ld_in, void* out_act, int out_f16, ActOut out_q,
           cudaStream_t st);

struct RopeKVArgs {
  const void* qkv;       // [T, (H + 2*Hkv) * D]  f32 or bf16
  int qkv_is_bf16;
  int ld_qkv;            // elements per token row
  const int* pos;        // [T]
  const int64_t* slots;  // [T] physical slot = block * block_size + offset (-1 = skip)
  const float* cos_t;    // [max_pos, rot/2]
  const float* sin_t;
  const float* q_norm;   // optional [D] (Qwen3 QK-norm)
  const float* k_norm;
  float norm_eps;
  int T, H, Hkv, D, rot, neox;
  __nv_bfloat16* q_out;  // [T, H, D]
  void* kcache;          // [num_blocks, Hkv, block_size, D] (fp16 or bf16)
  void* vcache;
  int cache_type;           // KV cache element type: kCacheF16, kCacheBF16 or kCacheFP8 (e4m3)
  int block_size;
  // fp8 cache: one f32 scale per stored row ([num_blocks, Hkv, block_size]); the row holds
  // e4m3(x / scale) with scale = max|x| / 448.  Null: unscaled e4m3.
  float* kscale = nullptr;
  float* vscale = nullptr;
};
int rope_kv_write(const RopeKVArgs& a, cudaStream_t st);

struct DecodeAttnArgs {
  const __nv_bfloat16* q;   // [B, H, D]
  const void* kcache;       // [num_blocks, Hkv, bs, D]
  const void* vcache;
  int cache_type;           // KV cache element type: kCacheF16, kCacheBF16 or kCacheFP8 (e4m3)
  const int* block_tables;  // [B, max_blocks]
  int max_blocks;
  const int* seq_lens;      // [B] tokens in cache including the current one
  int B, H, Hkv, D, block_size;
  float scale;
  int window;               // sliding window (0 = none)
  int splits;               // KV splits per (b, kv head)
  float* part_acc;          // scratch [B, Hkv, splits, G, D]
  float2* part_ml;          // scratch [B, Hkv, splits, G] (max, sum)
  void* out;                // [B, H*D] activation dtype
  int out_f16;
  ActOut out_q;             // optional q8 of out (q == null: none)
  // optional [B * Hkv] zeroed arrival counters: the last split CTA of a (b, kv head) merges the
  // splits itself (no second launch); null = a separate merge kernel
  int* counters = nullptr;
  const float* kscale = nullptr;  // fp8 cache: per-row scales (RopeKVArgs), null = unscaled
  const float* vscale = nullptr;
  // pages in the cache; a block-table entry outside [0, num_blocks) is recorded in *err (0xA00)
  // and read as page 0 instead.  0 = unchecked.
  int num_blocks = 0;
  int* err = nullptr;
};
int decode_attention(const DecodeAttnArgs& a, cudaStream_t st);
size_t decode_attention_scratch_floats(int B, int H, int Hkv, int D, int splits);

struct PrefillAttnArgs {
  const __nv_bfloat16* q;   // [T, H, D]  (rows of all sequences, concatenated)
  const void* kcache;
  const void* vcache;
  int cache_type;           // KV cache element type: kCacheF16, kCacheBF16 or kCacheFP8 (e4m3)
  const int* block_tables;  // [S, max_blocks]
  int max_blocks;
  const int* q_start;       // [S+1] prefix sums of new tokens per sequence
  const int* ctx_lens;      // [S] total tokens in cache after this step (prefix + new)
  int S, max_q, H, Hkv, D, block_size;
  float scale;
  int window;
  void* out;                // [T, H*D] activation dtype
  int out_f16;
  const float* kscale = nullptr;  // fp8 cache: per-row scales (RopeKVArgs), null = unscaled
  const float* vscale = nullptr;
  long cache_rows = 0;            // rows of the cache viewed as [blocks * Hkv * block_size, D] (tcgen05 path)
  int impl = 0;                   // 0: mma.sync kernel; 1: tcgen05 kernel where it has an instantiation
};
int prefill_attention(const PrefillAttnArgs& a, cudaStream_t st);
// The tcgen05 / TMEM / TMA kernel (attn_prefill_tc.cu): -2 when the cache type or D has no
// instantiation (fp8 caches, D other than 64 / 128).
int prefill_attention_tc(const PrefillAttnArgs& a, cudaStream_t st);

// Token embedding rows gathered from a quantized [V, H] table (planar layout) into f32 [T, H].
int embed_gather(const QW& table, const int* ids, int T, float* out, cudaStream_t st);

// Dequantize rows [r0, r0+n) of a quantized weight to bf16 [n, K] (used by the GEMM path tests
// and for types without a native kernel).
int dequant_rows(const QW& w, int r0, int n, __nv_bfloat16* out, cudaStream_t st);

struct SampleArgs {
  const float* logits;  // [B, V]
  int B, V, ld;
  const float* temperature;  // [B]  (<= 0 -> greedy)
  const int* top_k;          // [B]  (<= 0 -> off)
  const float* top_p;        // [B]  (>= 1 -> off)
  const float* min_p;        // [B]  (<= 0 -> off)
  const uint64_t* seeds;     // [B]
  const int* steps;          // [B] per-sequence offset into the Philox stream
  int* out_ids;              // [B]
  float* out_logprob;        // optional [B]
  const uint32_t* allow_mask;  // optional [B, ceil(V/32)] grammar bitmask (1 = allowed)
  const float* penalties;    // optional [B, 3] (repetition, frequency, presence)
  const int* pen_counts_idx; // optional [B, max_hist] token history (-1 padded)
  int max_hist;
};
int sample_tokens(const SampleArgs& a, cudaStream_t st);

// K14: speculative-decoding rejection step on the device (sampler.cu); out int32 [k + 2].
int spec_verify(const float* ps, const float* qs, const int64_t* drafts, int k, int V, int greedy, uint64_t seed,
                uint32_t step, int* out, cudaStream_t st);

}  // namespace barq
