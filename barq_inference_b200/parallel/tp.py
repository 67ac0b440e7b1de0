"""Tensor / expert parallel sharding of GGUF tensors (Megatron layout), straight from GGUF blocks.

Parity: ``TensorParallel::{column_parallel_linear,row_parallel_linear,parallel_attention}``
(``backend/src/cuda_multi_gpu.rs:255-328``, which documents the split but shards nothing) and
``advanced::TensorParallel::split_tensor`` (``advanced/src/tensor_parallel.rs:68-124``).

Per rank r of ``tp``:
  * column-parallel (output rows split): attn_q / attn_k / attn_v by heads, ffn_gate / ffn_up and the
    shared experts' gate/up by rows;
  * row-parallel (input columns split on quant-block boundaries): attn_output, ffn_down, shared
    down -- each rank produces a partial sum that an all-reduce completes;
  * expert parallel: the routed experts are split by expert (rank r holds experts
    [r*E/tp, (r+1)*E/tp)); the router is replicated and every rank routes all tokens;
  * vocab-parallel head: output rows split, logits all-gathered;
  * embeddings and norms are replicated.
Sharding works on the packed GGUF rows: a row shard selects rows, a column shard takes the byte
range of whole quant blocks in every row, so no weight is dequantized.
"""
from __future__ import annotations

import dataclasses

from ..gguf import TYPE_TRAITS
from ..models.config import ModelConfig
from ..models.weights import PackedTensor


@dataclasses.dataclass
class TPInfo:
    rank: int
    world: int
    expert0: int = 0       # first routed expert held by this rank
    n_experts_local: int = 0
    vocab0: int = 0        # first vocabulary row of this rank's head shard
    vocab_local: int = 0
    head0: int = 0         # MLA: first attention head of this rank
    n_heads_local: int = 0


def _rows(pt: PackedTensor, r0: int, n: int, shape: tuple[int, ...]) -> PackedTensor:
    return PackedTensor(pt.name, pt.ggml_type, shape, pt.data[r0:r0 + n].contiguous())


def _cols(pt: PackedTensor, k0: int, k1: int) -> PackedTensor:
    tr = TYPE_TRAITS[pt.ggml_type]
    if k0 % tr.block_size or k1 % tr.block_size:
        raise ValueError(f"{pt.name}: column shard [{k0},{k1}) not on {tr.block_size}-element blocks")
    b0, b1 = k0 // tr.block_size * tr.type_size, k1 // tr.block_size * tr.type_size
    shape = tuple(pt.shape[:-1]) + (k1 - k0,)
    return PackedTensor(pt.name, pt.ggml_type, shape, pt.data[:, b0:b1].contiguous())


def _split(n: int, world: int, rank: int, what: str) -> tuple[int, int]:
    if n % world:
        raise ValueError(f"tensor parallel: {what} ({n}) is not divisible by tp={world}")
    k = n // world
    return rank * k, k


def shard_config(cfg: ModelConfig, world: int) -> ModelConfig:
    """The per-rank model config: heads and FFN widths divided by ``world`` (experts stay global)."""
    return dataclasses.replace(cfg, n_heads=cfg.n_heads // world, n_kv_heads=cfg.n_kv_heads // world,
                               ffn=cfg.ffn // world,
                               shared_expert_ffn=(cfg.shared_expert_ffn or cfg.expert_ffn) // world
                               if cfg.n_shared_experts else cfg.shared_expert_ffn)


def shard_tensors(cfg: ModelConfig, tensors: dict[str, PackedTensor], rank: int, world: int
                  ) -> tuple[dict[str, PackedTensor], TPInfo]:
    """This rank's tensors for tensor parallelism of degree ``world`` (attention TP x MoE EP)."""
    if cfg.is_mla:
        return _shard_mla(cfg, tensors, rank, world)
    H, Hkv, D = cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    _split(H, world, rank, "attention heads")
    _split(Hkv, world, rank, "KV heads")
    info = TPInfo(rank, world)
    out: dict[str, PackedTensor] = {}
    for name, pt in tensors.items():
        short = name.split(".", 2)[-1] if name.startswith("blk.") else name
        if short in ("attn_q.bias", "attn_k.bias", "attn_v.bias"):  # 1-D: one GGUF row, slice its elements
            h0, hn = _split(H if short == "attn_q.bias" else Hkv, world, rank, "heads")
            out[name] = _cols(pt, h0 * D, (h0 + hn) * D)
        elif short == "attn_q.weight":
            h0, hn = _split(H, world, rank, "heads")
            out[name] = _rows(pt, h0 * D, hn * D, (hn * D,) + tuple(pt.shape[1:]))
        elif short in ("attn_k.weight", "attn_v.weight"):
            h0, hn = _split(Hkv, world, rank, "KV heads")
            out[name] = _rows(pt, h0 * D, hn * D, (hn * D,) + tuple(pt.shape[1:]))
        elif short in ("ffn_gate.weight", "ffn_up.weight", "ffn_gate_shexp.weight", "ffn_up_shexp.weight"):
            f0, fn = _split(pt.shape[0], world, rank, short)
            out[name] = _rows(pt, f0, fn, (fn,) + tuple(pt.shape[1:]))
        elif short in ("attn_output.weight", "ffn_down.weight", "ffn_down_shexp.weight"):
            k0, kn = _split(pt.shape[-1], world, rank, short)
            out[name] = _cols(pt, k0, k0 + kn)
        elif short in ("ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight"):
            E = pt.shape[0]
            e0, en = _split(E, world, rank, "experts")
            per = pt.rows // E
            out[name] = _rows(pt, e0 * per, en * per, (en,) + tuple(pt.shape[1:]))
            info.expert0, info.n_experts_local = e0, en
        elif (name == "output.weight" or (name == "token_embd.weight" and "output.weight" not in tensors)) \
                and pt.shape[0] % world == 0:
            V = pt.shape[0]
            vn = V // world
            v0 = rank * vn
            info.vocab0, info.vocab_local = v0, vn
            if name == "output.weight":
                out[name] = _rows(pt, v0, vn, (vn,) + tuple(pt.shape[1:]))
            else:  # tied embeddings: keep the full table for the lookup, add a head shard
                out[name] = pt
                out["output.weight"] = _rows(pt, v0, vn, (vn,) + tuple(pt.shape[1:]))
        else:
            out[name] = pt
    return out, info


def _shard_mla(cfg: ModelConfig, tensors: dict[str, PackedTensor], rank: int, world: int
               ) -> tuple[dict[str, PackedTensor], TPInfo]:
    """DeepSeek-V2 (MLA): attention heads split over the ranks, the latent path replicated.

    Per rank: the query projection rows and the per-head ``attn_kv_b`` blocks (W_UK / W_UV) of its
    heads; ``attn_output`` columns of its heads (row-parallel, completed by the all-reduce);
    ``attn_q_a`` / ``attn_kv_a_mqa`` and their norms whole, so every rank writes the same latent
    cache rows.  Routed experts split by expert and the head by vocabulary as for the dense models;
    the dense FFN and the shared experts replicated (added by rank 0 only)."""
    H, dn, dv, dr = cfg.n_heads, cfg.qk_nope_dim, cfg.v_head_dim, cfg.qk_rope_dim
    h0, hn = _split(H, world, rank, "attention heads")
    info = TPInfo(rank, world)
    out: dict[str, PackedTensor] = {}
    rest: dict[str, PackedTensor] = {}
    for name, pt in tensors.items():
        short = name.split(".", 2)[-1] if name.startswith("blk.") else name
        if short in ("attn_q.weight", "attn_q_b.weight"):
            qd = dn + dr
            out[name] = _rows(pt, h0 * qd, hn * qd, (hn * qd,) + tuple(pt.shape[1:]))
        elif short == "attn_kv_b.weight":
            kd = dn + dv
            out[name] = _rows(pt, h0 * kd, hn * kd, (hn * kd,) + tuple(pt.shape[1:]))
        elif short == "attn_output.weight":
            out[name] = _cols(pt, h0 * dv, (h0 + hn) * dv)
        elif short.startswith("attn_"):
            out[name] = pt  # q_a / kv_a projections, norms: replicated latent path
        elif short in ("ffn_gate.weight", "ffn_up.weight", "ffn_down.weight", "ffn_gate_shexp.weight",
                       "ffn_up_shexp.weight", "ffn_down_shexp.weight"):
            # the leading dense FFN and the shared experts stay whole (their widths, e.g. 10944 / 8,
            # do not split into the GEMM's 128-row tiles); rank 0 alone adds them to the partial sums
            out[name] = pt
        else:
            rest[name] = pt
    # FFNs (dense, shared experts, routed experts) and the vocabulary-parallel head: the dense rules
    dense_cfg = dataclasses.replace(cfg, kv_lora_rank=0, n_heads=world, n_kv_heads=world, head_dim=1)
    ffn, finfo = shard_tensors(dense_cfg, rest, rank, world)
    out.update(ffn)
    info.expert0, info.n_experts_local = finfo.expert0, finfo.n_experts_local
    info.vocab0, info.vocab_local = finfo.vocab0, finfo.vocab_local
    info.head0, info.n_heads_local = h0, hn
    return out, info
