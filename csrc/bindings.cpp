// Torch bindings for the barq sm_100a kernels.  Every op checks device, dtype and contiguity and
// raises on a bad launch status; there is no CPU or library fallback behind these entry points.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "kernels/launch.h"
#include "kernels/pdl.cuh"

using torch::Tensor;
using OptT = c10::optional<Tensor>;

namespace {

#define CHECK_CUDA(t) TORCH_CHECK((t).is_cuda() && (t).is_contiguous(), #t " must be a contiguous CUDA tensor")

template <typename T> T* ptr(const Tensor& t) { return reinterpret_cast<T*>(t.data_ptr()); }
template <typename T> T* optptr(const OptT& t) { return t.has_value() && t->defined() ? reinterpret_cast<T*>(t->data_ptr()) : nullptr; }

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check(int rc, const char* what) {
  TORCH_CHECK(rc == 0, what, ": launch rejected with status ", rc);
  cudaError_t e = cudaPeekAtLastError();
  TORCH_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e));
}

int is_f16(const OptT& t) { return t.has_value() && t->defined() && t->scalar_type() == torch::kHalf; }
int cache_type_of(const torch::Tensor& c) {
  if (c.scalar_type() == torch::kBFloat16) return barq::kCacheBF16;
  if (c.scalar_type() == torch::kFloat8_e4m3fn) return barq::kCacheFP8;
  TORCH_CHECK(c.scalar_type() == torch::kHalf, "KV cache must be float16, bfloat16 or float8_e4m3fn");
  return barq::kCacheF16;
}

barq::ActOut act_out(const OptT& q, const OptT& s, const OptT& ql, const OptT& dl) {
  return barq::ActOut{optptr<int8_t>(q), optptr<float2>(s), optptr<int8_t>(ql), optptr<float2>(dl)};
}

barq::QW make_qw(int64_t type, int64_t N, int64_t K, const Tensor& p0, const OptT& p1, const OptT& p2, const OptT& d) {
  CHECK_CUDA(p0);
  barq::QW w;
  w.p0 = ptr<const uint8_t>(p0);
  w.p1 = optptr<const uint8_t>(p1);
  w.p2 = optptr<const uint8_t>(p2);
  w.d = optptr<const uint16_t>(d);
  w.N = (int)N;
  w.K = (int)K;
  w.type = (int)type;
  return w;
}

void qgemv(int64_t type, int64_t N, int64_t K, Tensor p0, OptT p1, OptT p2, OptT d, OptT xq, OptT xs, OptT xql,
           OptT xdl, OptT xb, int64_t B, int64_t mode, OptT out_f32, OptT out_bf16, OptT out_q, OptT out_s,
           OptT out_ql, OptT out_dl, OptT bias, int64_t ld_out, OptT ws_acc, OptT ws_cnt, OptT norm_h, OptT norm_w,
           double norm_eps, int64_t norm_x2) {
  c10::cuda::CUDAGuard g(p0.device());
  barq::QW w = make_qw(type, N, K, p0, p1, p2, d);
  barq::ActQ8 x{optptr<const int8_t>(xq), optptr<const float2>(xs), optptr<const int8_t>(xql),
                optptr<const float2>(xdl)};
  barq::GemvEpi ep{(int)mode, optptr<float>(out_f32), optptr<__nv_bfloat16>(out_bf16),
                   act_out(out_q, out_s, out_ql, out_dl), optptr<const float>(bias), (int)ld_out};
  TORCH_CHECK(!norm_h || (ws_acc && ws_cnt), "qgemv: the fused norm needs the streaming kernel");
  if (ws_acc && ws_cnt && type != barq::W_BF16) {
    TORCH_CHECK(ws_acc->numel() >= barq::qgemv_stream_ws_floats((int)N) && ws_cnt->numel() >= (N + 127) / 128, "qgemv: workspace too small");
    check(barq::qgemv_stream(w, x, (int)B, ep, ptr<float>(*ws_acc), ptr<int>(*ws_cnt), barq::kernel_err_word(),
                             optptr<const float>(norm_h), optptr<const float>(norm_w), (float)norm_eps, (int)norm_x2,
                             cur_stream()),
          "qgemv_stream");
    return;
  }
  int ldxb = (int)K;
  check(barq::qgemv(w, x, optptr<const __nv_bfloat16>(xb), ldxb, (int)B, ep, cur_stream()), "qgemv");
}

void qgemm(int64_t type, int64_t N, int64_t K, Tensor p0, OptT p1, OptT p2, OptT d, Tensor x, int64_t T, int64_t mode,
           OptT out_f32, OptT out_bf16, OptT bias, int64_t ld_out, int64_t k_splits) {
  c10::cuda::CUDAGuard g(p0.device());
  const bool f16 = x.scalar_type() == torch::kHalf;
  TORCH_CHECK((f16 || x.scalar_type() == torch::kBFloat16) && x.is_contiguous() && x.size(-1) == K,
              "qgemm: x must be fp16 or bf16 [T, K]");
  if (out_bf16.has_value() && out_bf16->defined())
    TORCH_CHECK(out_bf16->scalar_type() == x.scalar_type(), "qgemm: activation output must have x's dtype");
  barq::QW w = make_qw(type, N, K, p0, p1, p2, d);
  barq::GemvEpi ep{(int)mode, optptr<float>(out_f32), optptr<__nv_bfloat16>(out_bf16), barq::ActOut{},
                   optptr<const float>(bias), (int)ld_out};
  check(barq::qgemm_tc(w, x.data_ptr(), f16, (int)T, ep, (int)k_splits, cur_stream()), "qgemm");
}

// Sequence-parallel TP GEMM (tp_fused.cu): mode EPI_RS_PUSH pushes each output tile into its owner's
// receive slots (rs_slots / rs_flags: int64 device addresses [world]); ag_flags (optional): the token
// tiles of x are loaded only after their gather flags reached *ag_epoch.
void qgemm_sp(int64_t type, int64_t N, int64_t K, Tensor p0, OptT p1, OptT p2, OptT d, Tensor x, int64_t T,
              int64_t mode, OptT out_f32, OptT out_bf16, OptT bias, int64_t ld_out, std::vector<int64_t> rs_slots,
              std::vector<int64_t> rs_flags, OptT rs_epoch, int64_t rank, int64_t chunk, int64_t max_tiles,
              OptT ag_flags, OptT ag_epoch, double wait_s) {
  c10::cuda::CUDAGuard g(p0.device());
  const bool f16 = x.scalar_type() == torch::kHalf;
  TORCH_CHECK((f16 || x.scalar_type() == torch::kBFloat16) && x.stride(-1) == 1 && x.size(-1) == K &&
                  (x.dim() == 1 || x.stride(0) == K),
              "qgemm_sp: x must be fp16 or bf16 [T, K], row-major");
  barq::QW w = make_qw(type, N, K, p0, p1, p2, d);
  barq::GemvEpi ep{(int)mode, optptr<float>(out_f32), optptr<__nv_bfloat16>(out_bf16), barq::ActOut{},
                   optptr<const float>(bias), (int)ld_out};
  barq::SpPush rs{};
  const barq::SpPush* prs = nullptr;
  if (mode == barq::EPI_RS_PUSH) {
    TORCH_CHECK(rs_slots.size() == rs_flags.size() && !rs_slots.empty() && rs_slots.size() <= (size_t)barq::kSpMaxRanks &&
                    rs_epoch.has_value(), "qgemm_sp: RS targets");
    for (size_t q = 0; q < rs_slots.size(); ++q) {
      rs.slots[q] = reinterpret_cast<float*>(rs_slots[q]);
      rs.flags[q] = reinterpret_cast<uint32_t*>(rs_flags[q]);
    }
    rs.epoch = reinterpret_cast<const uint32_t*>(rs_epoch->data_ptr());
    rs.rank = (int)rank;
    rs.world = (int)rs_slots.size();
    rs.chunk = (int)chunk;
    rs.max_tiles = (int)max_tiles;
    prs = &rs;
  }
  barq::SpWait agw{};
  const barq::SpWait* pagw = nullptr;
  if (ag_flags.has_value() && ag_flags->defined()) {
    TORCH_CHECK(ag_epoch.has_value(), "qgemm_sp: ag_epoch");
    agw.flags = reinterpret_cast<const uint32_t*>(ag_flags->data_ptr());
    agw.epoch = reinterpret_cast<const uint32_t*>(ag_epoch->data_ptr());
    agw.wait_ns = (unsigned long long)(wait_s * 1e9);
    pagw = &agw;
  }
  check(barq::qgemm_tc(w, x.data_ptr(), f16, (int)T, ep, 1, cur_stream(), nullptr, prs, pagw), "qgemm_sp");
}

// Owner side of a sequence-parallel site: x (this rank's residual rows, f32 [rows, H]) += sum over the
// received slots; RMSNorm -> bf16 rows pushed into every rank's gather buffer (ag / ag_flags:
// int64 device addresses [world]).  epoch / done: this site's int32 counters (one element each).
void sp_reduce_norm_ag(Tensor x, int64_t T, int64_t rank, int64_t chunk, OptT slots, OptT rs_flags, int64_t n_src,
                       int64_t max_tiles, int64_t gemm_bn, int64_t n_tiles, OptT bias, Tensor norm_w, double eps,
                       std::vector<int64_t> ag, std::vector<int64_t> ag_flags, Tensor epoch, Tensor done,
                       double wait_s, int64_t out_f16, int64_t self_only) {
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous(), "sp_reduce_norm_ag: x f32 contiguous");
  TORCH_CHECK(ag.size() == ag_flags.size() && !ag.empty() && ag.size() <= (size_t)barq::kSpMaxRanks,
              "sp_reduce_norm_ag: ranks");
  TORCH_CHECK(norm_w.scalar_type() == torch::kFloat32 && norm_w.numel() == x.size(-1), "sp_reduce_norm_ag: norm_w");
  barq::SpReduceArgs a{};
  a.slots = optptr<const float>(slots);
  a.rs_flags = optptr<const uint32_t>(rs_flags);
  a.n_src = (int)n_src;
  a.max_tiles = (int)max_tiles;
  a.gemm_bn = (int)gemm_bn;
  a.n_tiles = (int)n_tiles;
  a.bias = optptr<const float>(bias);
  a.x = ptr<float>(x);
  a.T = (int)T;
  a.W = (int)ag.size();
  a.rank = (int)rank;
  a.chunk = (int)chunk;
  a.H = (int)x.size(-1);
  a.norm_w = ptr<const float>(norm_w);
  a.eps = (float)eps;
  a.out_f16 = (int)out_f16;
  a.self_only = (int)self_only;
  for (size_t q = 0; q < ag.size(); ++q) {
    a.ag[q] = reinterpret_cast<void*>(ag[q]);
    a.ag_flags[q] = reinterpret_cast<uint32_t*>(ag_flags[q]);
  }
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr());
  a.done = ptr<int>(done);
  a.err = barq::kernel_err_word();
  a.wait_ns = (unsigned long long)(wait_s * 1e9);
  check(barq::sp_reduce_norm_ag(a, cur_stream()), "sp_reduce_norm_ag");
}

void sp_ag_wait(Tensor flags, Tensor epoch, int64_t T, double wait_s) {
  c10::cuda::CUDAGuard g(flags.device());
  check(barq::sp_ag_wait(reinterpret_cast<const uint32_t*>(flags.data_ptr()),
                         reinterpret_cast<const uint32_t*>(epoch.data_ptr()), (int)T, barq::kernel_err_word(),
                         (unsigned long long)(wait_s * 1e9), cur_stream()),
        "sp_ag_wait");
}

int64_t gemm_tile_rows(int64_t T) { return barq::gemm_tile_rows((int)T); }

// Grouped (MoE expert) GEMM: w holds ng groups of grows rows; x [Ttot, K] rows sorted by group.
void qgemm_grouped(int64_t type, int64_t N, int64_t K, Tensor p0, OptT p1, OptT p2, OptT d, Tensor x, int64_t T,
                   int64_t mode, OptT out_f32, OptT out_act, int64_t ld_out, Tensor off, int64_t ng, int64_t grows,
                   OptT row_tok, OptT row_w) {
  c10::cuda::CUDAGuard g(p0.device());
  const bool f16 = x.scalar_type() == torch::kHalf;
  TORCH_CHECK((f16 || x.scalar_type() == torch::kBFloat16) && x.is_contiguous() && x.size(-1) == K,
              "qgemm_grouped: x must be fp16 or bf16 [T, K]");
  TORCH_CHECK(off.scalar_type() == torch::kInt32 && off.numel() >= ng + 1, "qgemm_grouped: off must be int32 [ng+1]");
  barq::QW w = make_qw(type, N, K, p0, p1, p2, d);
  barq::GemvEpi ep{(int)mode, optptr<float>(out_f32), optptr<__nv_bfloat16>(out_act), barq::ActOut{}, nullptr,
                   (int)ld_out};
  barq::GemmGroups grp{ptr<const int>(off), (int)ng, (int)grows, optptr<const int>(row_tok),
                       optptr<const float>(row_w)};
  check(barq::qgemm_tc(w, x.data_ptr(), f16, (int)T, ep, 1, cur_stream(), &grp), "qgemm_grouped");
}

void moe_router_logits(Tensor x, Tensor w, Tensor out) {
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.dim() == 2 && (x.scalar_type() == torch::kHalf || x.scalar_type() == torch::kBFloat16) &&
                  x.stride(1) == 1, "moe_router_logits: x fp16/bf16 [T, H] with unit column stride");
  TORCH_CHECK(w.dim() == 2 && w.scalar_type() == torch::kFloat32 && w.is_contiguous() && w.size(1) == x.size(1),
              "moe_router_logits: w f32 [E, H] contiguous");
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous() && out.size(0) == x.size(0) &&
                  out.size(1) == w.size(0), "moe_router_logits: out f32 [T, E] contiguous");
  check(barq::moe_router_logits(x.data_ptr(), x.scalar_type() == torch::kHalf, (int)x.stride(0), ptr<const float>(w),
                                ptr<float>(out), (int)x.size(0), (int)w.size(0), (int)x.size(1), cur_stream()),
        "moe_router_logits");
}

void moe_route(Tensor logits, int64_t k, int64_t sigmoid, int64_t renorm, int64_t n_group, int64_t topk_group,
               double ser_threshold, double scale, Tensor x, Tensor ids, Tensor weights, Tensor counts, Tensor cursor,
               Tensor off, Tensor row_tok, Tensor row_w, Tensor tok_row, OptT xs) {
  c10::cuda::CUDAGuard g(logits.device());
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.dim() == 2, "moe_route: logits f32 [T, E]");
  TORCH_CHECK(x.scalar_type() == torch::kHalf || x.scalar_type() == torch::kBFloat16, "moe_route: x fp16/bf16");
  barq::MoeRouteArgs a;
  a.logits = ptr<const float>(logits);
  a.T = (int)logits.size(0);
  a.E = (int)logits.size(1);
  a.k = (int)k;
  a.H = (int)x.size(1);
  a.sigmoid = (int)sigmoid;
  a.renorm = (int)renorm;
  a.n_group = (int)n_group;
  a.topk_group = (int)topk_group;
  a.ser_threshold = (float)ser_threshold;
  a.scale = (float)scale;
  a.ids = ptr<int>(ids);
  a.weights = ptr<float>(weights);
  a.counts = ptr<int>(counts);
  a.cursor = ptr<int>(cursor);
  a.off = ptr<int>(off);
  a.row_tok = ptr<int>(row_tok);
  a.row_w = ptr<float>(row_w);
  TORCH_CHECK(tok_row.scalar_type() == torch::kInt32 && tok_row.numel() >= (int64_t)a.T * a.k, "moe_route: tok_row int32 [T*k]");
  a.tok_row = ptr<int>(tok_row);
  check(barq::moe_route(a, x.data_ptr(), x.scalar_type() == torch::kHalf, optptr<void>(xs), cur_stream()), "moe_route");
}

void moe_combine(Tensor ys, Tensor tok_row, Tensor lo, Tensor hi, int64_t T, int64_t k, Tensor x) {
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(ys.scalar_type() == torch::kFloat32 && x.scalar_type() == torch::kFloat32, "moe_combine: f32 ys and x");
  TORCH_CHECK(ys.stride(-1) == 1 && x.stride(-1) == 1 && ys.size(-1) >= x.size(-1), "moe_combine: row-major ys / x");
  TORCH_CHECK(tok_row.scalar_type() == torch::kInt32 && tok_row.numel() >= T * k, "moe_combine: tok_row int32 [T*k]");
  barq::MoeCombineArgs a{ptr<const float>(ys), (int)ys.stride(0), ptr<const int>(tok_row), ptr<const int>(lo),
                         ptr<const int>(hi), (int)T, (int)k, (int)x.size(1), ptr<float>(x), (int)x.stride(0)};
  check(barq::moe_combine(a, cur_stream()), "moe_combine");
}

// Expert-parallel all-to-all (moe.cu): which = 0 dispatch (counts exchange + row dispatch), 1 combine
// (signal + weighted gather into out).  Address lists hold every rank's buffer ([world] int64).
void ep_call(int64_t which, int64_t rank, int64_t E, int64_t E_local, int64_t k, int64_t rows, Tensor ids,
             Tensor weights, Tensor counts, Tensor cursor, std::vector<int64_t> cnt_all, std::vector<int64_t> cnt_flags,
             Tensor x, std::vector<int64_t> recv_x, std::vector<int64_t> disp_flags, Tensor disp_pos, Tensor recv_off,
             std::vector<int64_t> ys, std::vector<int64_t> ys_flags, OptT out, Tensor epoch, Tensor done, int64_t cap,
             double wait_s) {
  c10::cuda::CUDAGuard g(x.device());
  const size_t W = cnt_all.size();
  TORCH_CHECK(W >= 1 && W <= (size_t)barq::kSpMaxRanks && cnt_flags.size() == W && recv_x.size() == W &&
                  disp_flags.size() == W && ys.size() == W && ys_flags.size() == W, "ep_call: ranks");
  TORCH_CHECK(ids.scalar_type() == torch::kInt32 && weights.scalar_type() == torch::kFloat32 &&
                  ids.numel() >= rows * k && weights.numel() >= rows * k, "ep_call: routing");
  TORCH_CHECK(disp_pos.scalar_type() == torch::kInt32 && disp_pos.numel() >= 2 * rows * k, "ep_call: disp_pos");
  TORCH_CHECK(x.scalar_type() == torch::kHalf || x.scalar_type() == torch::kBFloat16, "ep_call: x fp16/bf16");
  barq::EpArgs a{};
  a.rank = (int)rank;
  a.W = (int)W;
  a.E = (int)E;
  a.E_local = (int)E_local;
  a.k = (int)k;
  a.H = (int)x.size(-1);
  a.rows = (int)rows;
  a.ids = ptr<const int>(ids);
  a.weights = ptr<const float>(weights);
  a.counts = ptr<int>(counts);
  a.cursor = ptr<int>(cursor);
  for (size_t q = 0; q < W; ++q) {
    a.cnt_all[q] = reinterpret_cast<int*>(cnt_all[q]);
    a.cnt_flags[q] = reinterpret_cast<uint32_t*>(cnt_flags[q]);
    a.recv_x[q] = reinterpret_cast<void*>(recv_x[q]);
    a.disp_flags[q] = reinterpret_cast<uint32_t*>(disp_flags[q]);
    a.ys[q] = reinterpret_cast<const float*>(ys[q]);
    a.ys_flags[q] = reinterpret_cast<uint32_t*>(ys_flags[q]);
  }
  a.x = x.data_ptr();
  a.disp_pos = reinterpret_cast<int2*>(disp_pos.data_ptr());
  a.recv_off = ptr<int>(recv_off);
  a.out = optptr<float>(out);
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr());
  a.done = ptr<int>(done);
  a.cap = (int)cap;
  a.err = barq::kernel_err_word();
  a.wait_ns = (unsigned long long)(wait_s * 1e9);
  if (which == 0)
    check(barq::ep_dispatch(a, x.scalar_type() == torch::kHalf, cur_stream()), "ep_dispatch");
  else {
    TORCH_CHECK(out.has_value() && out->scalar_type() == torch::kFloat32 && out->is_contiguous() &&
                    (rows == 0 || a.out), "ep_combine: out f32 [rows, H]");
    check(barq::ep_combine(a, cur_stream()), "ep_combine");
  }
}

void spec_verify(Tensor ps, OptT qs, Tensor drafts, int64_t greedy, int64_t seed, int64_t step, Tensor out) {
  c10::cuda::CUDAGuard g(ps.device());
  TORCH_CHECK(ps.scalar_type() == torch::kFloat32 && ps.is_contiguous() && ps.dim() == 2, "spec_verify: ps f32 [k+1, V]");
  const int64_t k = drafts.numel();
  TORCH_CHECK(ps.size(0) == k + 1 && drafts.scalar_type() == torch::kInt64, "spec_verify: ps rows / drafts");
  TORCH_CHECK(greedy || (qs.has_value() && qs->is_contiguous() && qs->scalar_type() == torch::kFloat32 &&
                         qs->size(0) >= k && qs->size(1) == ps.size(1)), "spec_verify: qs f32 [k, V]");
  TORCH_CHECK(out.scalar_type() == torch::kInt32 && out.numel() >= k + 2, "spec_verify: out int32 [k+2]");
  check(barq::spec_verify(ptr<const float>(ps), optptr<const float>(qs), ptr<const int64_t>(drafts), (int)k,
                          (int)ps.size(1), (int)greedy, (uint64_t)seed, (uint32_t)step, ptr<int>(out), cur_stream()),
        "spec_verify");
}

void mla_kv_write(Tensor kv_a, Tensor norm_w, double eps, Tensor cos, Tensor sin, int64_t neox, Tensor pos,
                  Tensor slots, Tensor cache, Tensor q, int64_t H, int64_t qdim, int64_t rope_off) {
  c10::cuda::CUDAGuard g(kv_a.device());
  TORCH_CHECK(kv_a.size(-1) == 576 && cache.size(-1) == 576, "mla_kv_write: latent rows are 576 wide");
  barq::MlaKvArgs a{ptr<const float>(kv_a), ptr<const float>(norm_w), (float)eps, ptr<const float>(cos),
                    ptr<const float>(sin), (int)neox, ptr<const int>(pos), ptr<const int64_t>(slots),
                    cache.data_ptr(), ptr<float>(q), (int)kv_a.size(0), (int)H, (int)qdim, (int)rope_off};
  check(barq::mla_kv_write(a, cache.scalar_type() == torch::kBFloat16, cur_stream()), "mla_kv_write");
}

int64_t mla_attn_scratch_floats(int64_t rows, int64_t splits) {
  return (int64_t)barq::mla_attn_scratch_floats((int)rows, (int)splits);
}

void mla_attention(Tensor q_lat, Tensor q, int64_t qdim, int64_t rope_off, Tensor cache, Tensor block_tables,
                   Tensor row_seq, Tensor row_len, int64_t H, int64_t splits, double scale, Tensor scratch,
                   Tensor o_lat, int64_t impl) {
  c10::cuda::CUDAGuard g(q_lat.device());
  const int rows = (int)q_lat.size(0);
  TORCH_CHECK((size_t)scratch.numel() >= barq::mla_attn_scratch_floats(rows, (int)splits), "mla: scratch too small");
  barq::MlaAttnArgs a;
  a.q_lat = ptr<const float>(q_lat);
  a.q_pe = ptr<const float>(q) + rope_off;
  a.q_pe_stride = (int)qdim;
  a.cache = cache.data_ptr();
  a.block_tables = ptr<const int>(block_tables);
  a.max_blocks = (int)block_tables.size(1);
  a.row_seq = ptr<const int>(row_seq);
  a.row_len = ptr<const int>(row_len);
  a.rows = rows;
  a.H = (int)H;
  a.splits = (int)splits;
  a.scale = (float)scale;
  a.part_acc = ptr<float>(scratch);
  a.part_ml = reinterpret_cast<float2*>(ptr<float>(scratch) + (size_t)rows * splits * H * 512);
  a.o_lat = ptr<float>(o_lat);
  a.err = barq::kernel_err_word();
  a.num_blocks = (int)cache.size(0);
  check(barq::mla_attention(a, cache.scalar_type() == torch::kBFloat16, cur_stream(), (int)impl), "mla_attention");
}

// bufs / flags: device addresses (one per rank) of the partial buffers and flag areas.
void allreduce_add(Tensor x, std::vector<int64_t> bufs, std::vector<int64_t> flags, Tensor epoch, int64_t rank,
                   int64_t blocks, double wait_s, int64_t skip_signal, int64_t mc) {
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous(), "allreduce_add: x must be contiguous f32");
  TORCH_CHECK(bufs.size() == flags.size() && bufs.size() <= (size_t)barq::kArMaxRanks, "allreduce_add: ranks");
  barq::ArArgs a{};
  a.x = ptr<float>(x);
  for (size_t r = 0; r < bufs.size(); ++r) {
    a.bufs[r] = reinterpret_cast<const float*>(bufs[r]);
    a.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);
  }
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr());
  a.err = barq::kernel_err_word();
  a.rank = (int)rank;
  a.world = (int)bufs.size();
  a.n = (int)x.numel();
  a.blocks = (int)blocks;
  a.wait_ns = (unsigned long long)(wait_s * 1e9);
  a.skip_signal = (int)skip_signal;
  a.mc = reinterpret_cast<float*>(mc);  // 0: peer-load form
  check(barq::allreduce_add(a, cur_stream()), "allreduce_add");
}

// Row-parallel GEMV with the tensor-parallel all-reduce fused in (EPI_AR_PUSH): x += sum over ranks
// of W_r a_r.  bufs: int64 device tensor [world] of every rank's receive-buffer address for this
// call site (each [world][B][N] 64-bit words);
// epoch / done: this rank's int32 [2] counters, indexed by j.
void qgemv_ar(int64_t type, int64_t N, int64_t K, Tensor p0, OptT p1, OptT p2, OptT d, OptT xq, OptT xs, OptT xql,
              OptT xdl, int64_t B, OptT bias, Tensor ws_acc, Tensor ws_cnt, Tensor x, Tensor bufs, Tensor epoch,
              Tensor done, int64_t j, int64_t rank, double wait_s, int64_t skip_signal) {
  c10::cuda::CUDAGuard g(p0.device());
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.stride(1) == 1 && x.size(0) >= B && x.size(1) == N,
              "qgemv_ar: x must be f32 [B, N] with unit column stride");
  TORCH_CHECK(bufs.is_cuda() && bufs.scalar_type() == torch::kInt64 && bufs.numel() >= 1 &&
                  bufs.numel() <= barq::kArMaxRanks && j >= 0 && j < 2,
              "qgemv_ar: ranks / buffer index");
  TORCH_CHECK(epoch.scalar_type() == torch::kInt32 && done.scalar_type() == torch::kInt32 && epoch.numel() >= 2 &&
                  done.numel() >= 2, "qgemv_ar: epoch / done must be int32 [2]");
  TORCH_CHECK(ws_acc.numel() >= barq::qgemv_stream_ws_floats((int)N) && ws_cnt.numel() >= (N + 127) / 128, "qgemv_ar: workspace too small");
  barq::QW w = make_qw(type, N, K, p0, p1, p2, d);
  barq::ActQ8 xa{optptr<const int8_t>(xq), optptr<const float2>(xs), optptr<const int8_t>(xql),
                 optptr<const float2>(xdl)};
  barq::GemvEpi ep{barq::EPI_AR_PUSH, nullptr, nullptr, barq::ActOut{}, optptr<const float>(bias), (int)N};
  barq::ArPush ar{};
  ar.dst = reinterpret_cast<uint64_t* const*>(bufs.data_ptr());
  ar.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr<int>()) + j;
  ar.done = done.data_ptr<int>() + j;
  ar.x = ptr<float>(x);
  ar.ld_x = (int)x.stride(0);
  ar.rank = (int)rank;
  ar.world = (int)bufs.numel();
  ar.skip_signal = (int)skip_signal;
  ar.wait_ns = (unsigned long long)(wait_s * 1e9);
  check(barq::qgemv_stream(w, xa, (int)B, ep, ptr<float>(ws_acc), ptr<int>(ws_cnt), barq::kernel_err_word(), nullptr,
                           nullptr, 0.f, 0, cur_stream(), &ar),
        "qgemv_ar");
}

void dequant_dense(int64_t type, int64_t N, int64_t K, Tensor p0, OptT p1, OptT p2, OptT d, Tensor out) {
  c10::cuda::CUDAGuard g(p0.device());
  TORCH_CHECK(out.is_contiguous() && out.numel() >= N * K &&
                  (out.scalar_type() == torch::kHalf || out.scalar_type() == torch::kBFloat16),
              "dequant_dense: out must be contiguous fp16/bf16 [N, K]");
  barq::QW w = make_qw(type, N, K, p0, p1, p2, d);
  check(barq::dequant_dense(w, out.data_ptr(), out.scalar_type() == torch::kHalf, cur_stream()), "dequant_dense");
}

int64_t gemm_error() {
  int v = 0;
  TORCH_CHECK(barq::gemm_error_word(&v) == 0, "gemm_error: read failed");
  return v;
}

void gemm_clear_error() { TORCH_CHECK(barq::gemm_clear_error_word() == 0, "gemm_clear_error failed"); }

void rmsnorm(Tensor x, OptT add, Tensor w, double eps, OptT out_bf16, OptT out_q, OptT out_s, OptT out_ql,
             OptT out_dl) {
  CHECK_CUDA(x);
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.scalar_type() == torch::kFloat32, "rmsnorm: residual stream must be f32");
  int H = (int)x.size(-1), T = (int)(x.numel() / H);
  check(barq::rmsnorm(ptr<float>(x), optptr<const float>(add), ptr<const float>(w), (float)eps, T, H,
                      optptr<void>(out_bf16), is_f16(out_bf16), act_out(out_q, out_s, out_ql, out_dl), cur_stream()),
        "rmsnorm");
}

void quantize_q8(Tensor x, int64_t T, int64_t H, int64_t ldx, OptT out_q, OptT out_s, OptT out_ql, OptT out_dl) {
  c10::cuda::CUDAGuard g(x.device());
  check(barq::quantize_q8(x.data_ptr(), x.scalar_type() == torch::kBFloat16, (int)T, (int)H, (int)ldx,
                          act_out(out_q, out_s, out_ql, out_dl), cur_stream()),
        "quantize_q8");
}

void swiglu(Tensor in, int64_t T, int64_t F, int64_t ld_in, OptT out_bf16, OptT out_q, OptT out_s, OptT out_ql,
            OptT out_dl) {
  c10::cuda::CUDAGuard g(in.device());
  check(barq::swiglu(in.data_ptr(), in.scalar_type() == torch::kBFloat16, (int)T, (int)F, (int)ld_in,
                     optptr<void>(out_bf16), is_f16(out_bf16), act_out(out_q, out_s, out_ql, out_dl), cur_stream()),
        "swiglu");
}

void rope_kv_write(Tensor qkv, int64_t ld_qkv, Tensor pos, OptT slots, Tensor cos_t, Tensor sin_t, OptT q_norm,
                   OptT k_norm, double norm_eps, int64_t T, int64_t H, int64_t Hkv, int64_t D, int64_t rot,
                   bool neox, Tensor q_out, Tensor kcache, Tensor vcache, OptT kscale, OptT vscale) {
  c10::cuda::CUDAGuard g(qkv.device());
  barq::RopeKVArgs a;
  a.qkv = qkv.data_ptr();
  a.qkv_is_bf16 = qkv.scalar_type() == torch::kBFloat16;
  a.ld_qkv = (int)ld_qkv;
  a.pos = ptr<const int>(pos);
  a.slots = optptr<const int64_t>(slots);
  a.cos_t = ptr<const float>(cos_t);
  a.sin_t = ptr<const float>(sin_t);
  a.q_norm = optptr<const float>(q_norm);
  a.k_norm = optptr<const float>(k_norm);
  a.norm_eps = (float)norm_eps;
  a.T = (int)T; a.H = (int)H; a.Hkv = (int)Hkv; a.D = (int)D; a.rot = (int)rot; a.neox = neox;
  a.q_out = ptr<__nv_bfloat16>(q_out);
  a.kcache = kcache.data_ptr();
  a.vcache = vcache.data_ptr();
  a.cache_type = cache_type_of(kcache);
  a.block_size = (int)kcache.size(-2);
  a.kscale = optptr<float>(kscale);
  a.vscale = optptr<float>(vscale);
  check(barq::rope_kv_write(a, cur_stream()), "rope_kv_write");
}

void decode_attention(Tensor q, Tensor kcache, Tensor vcache, Tensor block_tables, Tensor seq_lens, int64_t B,
                      int64_t H, int64_t Hkv, int64_t D, double scale, int64_t window, int64_t splits, Tensor scratch,
                      Tensor out, OptT out_q, OptT out_s, OptT out_ql, OptT out_dl, OptT counters, OptT kscale,
                      OptT vscale) {
  c10::cuda::CUDAGuard g(q.device());
  TORCH_CHECK(scratch.scalar_type() == torch::kFloat32, "scratch must be f32");
  TORCH_CHECK(!counters || (counters->scalar_type() == torch::kInt32 && counters->numel() >= B * Hkv),
              "decode_attention: counters must be int32 [>= B * Hkv] (zero)");
  size_t need = barq::decode_attention_scratch_floats((int)B, (int)H, (int)Hkv, (int)D, (int)splits);
  TORCH_CHECK((size_t)scratch.numel() >= need, "decode_attention: scratch too small (", scratch.numel(), " < ", need, ")");
  barq::DecodeAttnArgs a;
  a.q = ptr<const __nv_bfloat16>(q);
  a.kcache = kcache.data_ptr();
  a.vcache = vcache.data_ptr();
  a.cache_type = cache_type_of(kcache);
  a.block_tables = ptr<const int>(block_tables);
  a.max_blocks = (int)block_tables.size(1);
  a.seq_lens = ptr<const int>(seq_lens);
  a.B = (int)B; a.H = (int)H; a.Hkv = (int)Hkv; a.D = (int)D;
  a.block_size = (int)kcache.size(-2);
  a.scale = (float)scale;
  a.window = (int)window;
  a.splits = (int)splits;
  a.part_acc = ptr<float>(scratch);
  a.part_ml = reinterpret_cast<float2*>(ptr<float>(scratch) + (size_t)B * H * splits * D);
  a.kscale = optptr<const float>(kscale);
  a.vscale = optptr<const float>(vscale);
  a.num_blocks = (int)kcache.size(0);
  a.err = barq::kernel_err_word();
  a.out = out.data_ptr();
  a.out_f16 = out.scalar_type() == torch::kHalf;
  a.out_q = act_out(out_q, out_s, out_ql, out_dl);
  a.counters = optptr<int>(counters);
  check(barq::decode_attention(a, cur_stream()), "decode_attention");
}

void prefill_attention(Tensor q, Tensor kcache, Tensor vcache, Tensor block_tables, Tensor q_start, Tensor ctx_lens,
                       int64_t S, int64_t max_q, int64_t H, int64_t Hkv, int64_t D, double scale, int64_t window,
                       Tensor out, OptT kscale, OptT vscale, int64_t impl) {
  c10::cuda::CUDAGuard g(q.device());
  barq::PrefillAttnArgs a;
  a.q = ptr<const __nv_bfloat16>(q);
  a.kcache = kcache.data_ptr();
  a.vcache = vcache.data_ptr();
  a.cache_type = cache_type_of(kcache);
  a.block_tables = ptr<const int>(block_tables);
  a.max_blocks = (int)block_tables.size(1);
  a.q_start = ptr<const int>(q_start);
  a.ctx_lens = ptr<const int>(ctx_lens);
  a.S = (int)S; a.max_q = (int)max_q; a.H = (int)H; a.Hkv = (int)Hkv; a.D = (int)D;
  a.block_size = (int)kcache.size(-2);
  a.scale = (float)scale;
  a.window = (int)window;
  a.out = out.data_ptr();
  a.out_f16 = out.scalar_type() == torch::kHalf;
  a.kscale = optptr<const float>(kscale);
  a.vscale = optptr<const float>(vscale);
  if (impl == 1)
    TORCH_CHECK(kcache.is_contiguous() && vcache.is_contiguous() && kcache.sizes() == vcache.sizes(),
                "prefill_attention: the tcgen05 path reads K / V as contiguous [blocks, Hkv, 16, D] caches");
  a.cache_rows = (long)(kcache.numel() / D);
  a.impl = (int)impl;
  check(barq::prefill_attention(a, cur_stream()), "prefill_attention");
}

void embed_gather(int64_t type, int64_t N, int64_t K, Tensor p0, OptT p1, OptT p2, OptT d, Tensor ids, Tensor out) {
  c10::cuda::CUDAGuard g(p0.device());
  barq::QW w = make_qw(type, N, K, p0, p1, p2, d);
  check(barq::embed_gather(w, ptr<const int>(ids), (int)ids.numel(), ptr<float>(out), cur_stream()), "embed_gather");
}

void dequant_rows(int64_t type, int64_t N, int64_t K, Tensor p0, OptT p1, OptT p2, OptT d, int64_t r0, int64_t n,
                  Tensor out) {
  c10::cuda::CUDAGuard g(p0.device());
  barq::QW w = make_qw(type, N, K, p0, p1, p2, d);
  check(barq::dequant_rows(w, (int)r0, (int)n, ptr<__nv_bfloat16>(out), cur_stream()), "dequant_rows");
}

void sample(Tensor logits, int64_t B, int64_t V, Tensor temperature, Tensor top_k, Tensor top_p, Tensor min_p,
            Tensor seeds, Tensor steps, Tensor out_ids, OptT out_logprob, OptT allow_mask, OptT penalties,
            OptT history) {
  c10::cuda::CUDAGuard g(logits.device());
  barq::SampleArgs a;
  a.logits = ptr<const float>(logits);
  a.B = (int)B; a.V = (int)V; a.ld = (int)logits.size(-1);
  a.temperature = ptr<const float>(temperature);
  a.top_k = ptr<const int>(top_k);
  a.top_p = ptr<const float>(top_p);
  a.min_p = ptr<const float>(min_p);
  a.seeds = reinterpret_cast<const uint64_t*>(seeds.data_ptr());
  a.steps = ptr<const int>(steps);
  a.out_ids = ptr<int>(out_ids);
  a.out_logprob = optptr<float>(out_logprob);
  a.allow_mask = optptr<const uint32_t>(allow_mask);
  a.penalties = optptr<const float>(penalties);
  a.pen_counts_idx = optptr<const int>(history);
  a.max_hist = history.has_value() ? (int)history->size(-1) : 0;
  check(barq::sample_tokens(a, cur_stream()), "sample");
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "barq sm_100a kernels";
  m.def("qgemv", &qgemv);
  m.def("rmsnorm", &rmsnorm);
  m.def("qgemm", &qgemm);
  m.def("gemm_error", &gemm_error);
  m.def("qgemm_grouped", &qgemm_grouped);
  m.def("moe_route", &moe_route);
  m.def("moe_router_logits", &moe_router_logits);
  m.def("moe_combine", &moe_combine);
  m.def("ep_call", &ep_call);
  m.def("spec_verify", &spec_verify);
  m.def("qgemm_sp", &qgemm_sp);
  m.def("sp_reduce_norm_ag", &sp_reduce_norm_ag);
  m.def("sp_ag_wait", &sp_ag_wait);
  m.def("gemm_tile_rows", &gemm_tile_rows);
  m.def("mla_kv_write", &mla_kv_write);
  m.def("allreduce_add", &allreduce_add);
  m.def("qgemv_ar", &qgemv_ar);
  m.def("dequant_dense", &dequant_dense);
  m.def("set_pdl_mode", [](int64_t m) { barq::set_pdl_mode((int)m); });
  m.def("mla_attn_scratch_floats", &mla_attn_scratch_floats);
  m.def("mla_attention", &mla_attention);
  m.def("gemm_clear_error", &gemm_clear_error);
  m.def("gemm_set_trace", [](Tensor t) { barq::gemm_set_trace(t.data_ptr()); });
  m.def("quantize_q8", &quantize_q8);
  m.def("swiglu", &swiglu);
  m.def("rope_kv_write", &rope_kv_write);
  m.def("decode_attention", &decode_attention);
  m.def("decode_attention_scratch_floats", [](int64_t B, int64_t H, int64_t Hkv, int64_t D, int64_t s) {
    return (int64_t)barq::decode_attention_scratch_floats((int)B, (int)H, (int)Hkv, (int)D, (int)s);
  });
  m.def("prefill_attention", &prefill_attention);
  m.def("embed_gather", &embed_gather);
  m.def("dequant_rows", &dequant_rows);
  m.def("sample", &sample);
}
