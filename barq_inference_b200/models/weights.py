"""GGUF tensor naming per architecture, random-init checkpoints and config <-> metadata.

Tensor names follow llama.cpp's GGUF conventions (``blk.{i}.attn_q.weight`` ...), which is also what
the reference's ``WeightCache`` looks up (``models/src/weight_cache.rs:48-210``).  The random-init
generator replaces the reference's metadata-only fixtures (``models/src/test_support.rs:17-44``) with
complete checkpoints for every benchmark configuration.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Iterator

import numpy as np
import torch

from ..gguf import GGUFValueType, GGMLType, GGUFWriter, quantize
from ..gguf.ik_quants import IK_TYPES
from .config import ModelConfig


@dataclass
class QuantPolicy:
    """Which ggml type each class of tensor is stored in."""

    default: GGMLType = GGMLType.Q4_K
    attn: GGMLType | None = None  # attention projections (q/k/v/o and MLA)
    output: GGMLType | None = GGMLType.Q6_K
    embed: GGMLType | None = None
    experts: GGMLType | None = None
    router: GGMLType = GGMLType.F32
    norm: GGMLType = GGMLType.F32

    def type_for(self, kind: str) -> GGMLType:
        if kind == "norm" or kind == "bias":
            return self.norm
        if kind == "router":
            return self.router
        if kind == "output":
            return self.output or self.default
        if kind == "embed":
            return self.embed or self.default
        if kind == "attn":
            return self.attn or self.default
        if kind == "expert":
            return self.experts or self.default
        return self.default


POLICIES = {
    "tiny": QuantPolicy(default=GGMLType.Q4_0, output=GGMLType.Q8_0, embed=GGMLType.Q8_0),
    "tiny-ds": QuantPolicy(default=GGMLType.Q4_K, attn=GGMLType.Q8_0, output=GGMLType.Q8_0, embed=GGMLType.Q8_0),
    "tiny-moe": QuantPolicy(default=GGMLType.Q4_K, output=GGMLType.Q8_0, embed=GGMLType.Q8_0),
    "llama3-8b": QuantPolicy(default=GGMLType.Q4_K, output=GGMLType.Q6_K),
    "llama3-70b": QuantPolicy(default=GGMLType.Q4_K, attn=GGMLType.Q6_K, output=GGMLType.Q6_K),
    "mixtral-8x7b": QuantPolicy(default=GGMLType.Q4_K, output=GGMLType.Q6_K),
    "deepseek-v2-lite": QuantPolicy(default=GGMLType.Q4_K, attn=GGMLType.Q8_0, output=GGMLType.Q6_K),
}


def fallback_type(t: GGMLType, row_len: int) -> GGMLType:
    """Rows not divisible by the block size cannot be stored blocked; like llama.cpp's quantizer,
    fall back to a smaller block (32) and then to F16 (e.g. the tiny config's FFN width 688)."""
    from ..gguf import TYPE_TRAITS

    if row_len % TYPE_TRAITS[t].block_size == 0:
        return t
    if row_len % 32 == 0:
        return {GGMLType.Q6_K: GGMLType.Q8_0, GGMLType.Q5_K: GGMLType.Q5_0, GGMLType.IQ4_KS: GGMLType.IQ4_NL}.get(
            t, GGMLType.Q4_0 if t != GGMLType.Q8_0 else t)
    return GGMLType.F16


def tensor_plan(cfg: ModelConfig) -> Iterator[tuple[str, tuple[int, ...], str]]:
    """Yield (name, row-major shape, kind) for every tensor of the architecture."""
    h = cfg.hidden
    yield "token_embd.weight", (cfg.vocab, h), "embed"
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        yield p + "attn_norm.weight", (h,), "norm"
        if cfg.is_mla:
            qh = cfg.qk_nope_dim + cfg.qk_rope_dim
            if cfg.q_lora_rank:
                yield p + "attn_q_a.weight", (cfg.q_lora_rank, h), "attn"
                yield p + "attn_q_a_norm.weight", (cfg.q_lora_rank,), "norm"
                yield p + "attn_q_b.weight", (cfg.n_heads * qh, cfg.q_lora_rank), "attn"
            else:
                yield p + "attn_q.weight", (cfg.n_heads * qh, h), "attn"
            yield p + "attn_kv_a_mqa.weight", (cfg.kv_lora_rank + cfg.qk_rope_dim, h), "attn"
            yield p + "attn_kv_a_norm.weight", (cfg.kv_lora_rank,), "norm"
            yield p + "attn_kv_b.weight", (cfg.n_heads * (cfg.qk_nope_dim + cfg.v_head_dim), cfg.kv_lora_rank), "attn"
            yield p + "attn_output.weight", (h, cfg.n_heads * cfg.v_head_dim), "attn"
        else:
            yield p + "attn_q.weight", (cfg.q_dim, h), "attn"
            yield p + "attn_k.weight", (cfg.kv_dim, h), "attn"
            yield p + "attn_v.weight", (cfg.kv_dim, h), "attn"
            if cfg.qkv_bias:
                yield p + "attn_q.bias", (cfg.q_dim,), "bias"
                yield p + "attn_k.bias", (cfg.kv_dim,), "bias"
                yield p + "attn_v.bias", (cfg.kv_dim,), "bias"
            if cfg.qk_norm:
                yield p + "attn_q_norm.weight", (cfg.head_dim,), "norm"
                yield p + "attn_k_norm.weight", (cfg.head_dim,), "norm"
            yield p + "attn_output.weight", (h, cfg.q_dim), "attn"
        yield p + "ffn_norm.weight", (h,), "norm"
        if cfg.layer_is_moe(i):
            e, f = cfg.n_experts, cfg.expert_ffn
            yield p + "ffn_gate_inp.weight", (e, h), "router"
            yield p + "ffn_gate_exps.weight", (e, f, h), "expert"
            yield p + "ffn_up_exps.weight", (e, f, h), "expert"
            yield p + "ffn_down_exps.weight", (e, h, f), "expert"
            if cfg.n_shared_experts:
                fs = (cfg.shared_expert_ffn or cfg.expert_ffn) * cfg.n_shared_experts
                yield p + "ffn_gate_shexp.weight", (fs, h), "ffn"
                yield p + "ffn_up_shexp.weight", (fs, h), "ffn"
                yield p + "ffn_down_shexp.weight", (h, fs), "ffn"
        else:
            yield p + "ffn_gate.weight", (cfg.ffn, h), "ffn"
            yield p + "ffn_up.weight", (cfg.ffn, h), "ffn"
            yield p + "ffn_down.weight", (h, cfg.ffn), "ffn"
    yield "output_norm.weight", (h,), "norm"
    if not cfg.tied_embeddings:
        yield "output.weight", (cfg.vocab, h), "output"


def config_metadata(cfg: ModelConfig, name: str = "barq-random") -> dict:
    a = cfg.arch
    md = {
        "general.architecture": a,
        "general.name": name,
        f"{a}.block_count": cfg.n_layers,
        f"{a}.context_length": cfg.max_ctx,
        f"{a}.embedding_length": cfg.hidden,
        f"{a}.feed_forward_length": cfg.ffn,
        f"{a}.attention.head_count": cfg.n_heads,
        f"{a}.attention.head_count_kv": cfg.n_kv_heads,
        f"{a}.attention.layer_norm_rms_epsilon": float(cfg.rms_eps),
        f"{a}.rope.freq_base": float(cfg.rope_theta),
        f"{a}.vocab_size": cfg.vocab,
        "tokenizer.ggml.bos_token_id": cfg.bos_id,
        "tokenizer.ggml.eos_token_id": cfg.eos_ids[0],
    }
    if len(cfg.eos_ids) > 1:
        md["tokenizer.ggml.eot_token_id"] = cfg.eos_ids[1]
    if cfg.rope_dim:
        md[f"{a}.rope.dimension_count"] = cfg.rope_dim
    if cfg.rope_scaling != "none":
        md[f"{a}.rope.scaling.type"] = cfg.rope_scaling
        md[f"{a}.rope.scaling.factor"] = float(cfg.rope_factor)
        md[f"{a}.rope.scaling.original_context_length"] = cfg.rope_orig_ctx
        if cfg.yarn_log_mul:
            md[f"{a}.rope.scaling.yarn_log_multiplier"] = float(cfg.yarn_log_mul)
    if cfg.sliding_window:
        md[f"{a}.attention.sliding_window"] = cfg.sliding_window
    if cfg.is_moe:
        md[f"{a}.expert_count"] = cfg.n_experts
        md[f"{a}.expert_used_count"] = cfg.n_experts_used
        md[f"{a}.expert_feed_forward_length"] = cfg.expert_ffn
        if cfg.n_shared_experts:
            md[f"{a}.expert_shared_count"] = cfg.n_shared_experts
        if cfg.n_dense_layers:
            md[f"{a}.leading_dense_block_count"] = cfg.n_dense_layers
        md[f"{a}.expert_weights_scale"] = float(cfg.expert_weights_scale)
        md[f"{a}.expert_weights_norm"] = bool(cfg.expert_weights_norm)
    if cfg.is_mla:
        md[f"{a}.attention.kv_lora_rank"] = cfg.kv_lora_rank
        if cfg.q_lora_rank:
            md[f"{a}.attention.q_lora_rank"] = cfg.q_lora_rank
        md[f"{a}.attention.key_length"] = cfg.qk_nope_dim + cfg.qk_rope_dim
        md[f"{a}.attention.value_length"] = cfg.v_head_dim
        md[f"{a}.rope.dimension_count"] = cfg.qk_rope_dim
    return md


@dataclass
class PackedTensor:
    """One GGUF tensor: packed bytes (torch uint8, any device) + type + row-major shape."""

    name: str
    ggml_type: GGMLType
    shape: tuple[int, ...]
    data: torch.Tensor  # uint8, shape (prod(shape[:-1]), row_bytes)

    @property
    def rows(self) -> int:
        return int(np.prod(self.shape[:-1])) if len(self.shape) > 1 else 1

    @property
    def cols(self) -> int:
        return self.shape[-1]


def random_tensors(cfg: ModelConfig, policy: QuantPolicy, seed: int = 0, device: str | torch.device = "cpu",
                   std: float = 0.02, chunk_rows: int = 16384) -> dict[str, PackedTensor]:
    """N(0, std) weights from one generator seeded with ``seed`` (plan order), norms = 1."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    out: dict[str, PackedTensor] = {}
    for name, shape, kind in tensor_plan(cfg):
        t = policy.type_for(kind)
        if kind == "norm":
            w = torch.ones(shape, dtype=torch.float32, device=device)
            out[name] = PackedTensor(name, t, shape, quantize(w.reshape(1, -1), t))
            continue
        if kind == "bias":
            w = torch.randn(shape, generator=gen, device=device) * std
            out[name] = PackedTensor(name, t, shape, quantize(w.reshape(1, -1), t))
            continue
        rows = int(np.prod(shape[:-1]))
        k = shape[-1]
        t = fallback_type(t, k)
        parts = []
        for r0 in range(0, rows, chunk_rows):
            r = min(chunk_rows, rows - r0)
            w = torch.randn((r, k), generator=gen, device=device, dtype=torch.float32) * std
            parts.append(quantize(w, t))
        out[name] = PackedTensor(name, t, shape, torch.cat(parts, 0) if len(parts) > 1 else parts[0])
    return out


def write_gguf(path: str, cfg: ModelConfig, tensors: dict[str, PackedTensor], extra_md: dict | None = None) -> None:
    w = GGUFWriter(path)
    for k, v in config_metadata(cfg).items():
        w.add(k, v)
    for k, v in (extra_md or {}).items():
        w.add(k, v)
    for name, pt in tensors.items():
        w.add_tensor(name, pt.data.cpu().numpy(), pt.ggml_type, pt.shape)
    w.write()


def write_gguf_split(path: str, cfg: ModelConfig, tensors: dict[str, PackedTensor], n_parts: int,
                     extra_md: dict | None = None) -> list[str]:
    """Write ``path`` as ``n_parts`` files ``<base>-0000i-of-0000N.gguf`` (llama.cpp gguf-split layout:
    every part carries ``split.no`` / ``split.count`` / ``split.tensors.count``, the first one the
    model metadata, tensors distributed in order).  Returns the part paths."""
    base = path[:-5] if path.endswith(".gguf") else path
    names = list(tensors)
    per = (len(names) + n_parts - 1) // n_parts
    paths = []
    for i in range(n_parts):
        pp = f"{base}-{i + 1:05d}-of-{n_parts:05d}.gguf"
        w = GGUFWriter(pp)
        if i == 0:
            for k, v in config_metadata(cfg).items():
                w.add(k, v)
            for k, v in (extra_md or {}).items():
                w.add(k, v)
        w.add("split.no", i, GGUFValueType.UINT16)
        w.add("split.count", n_parts, GGUFValueType.UINT16)
        w.add("split.tensors.count", len(names), GGUFValueType.INT32)
        for name in names[i * per:(i + 1) * per]:
            pt = tensors[name]
            w.add_tensor(name, pt.data.cpu().numpy(), pt.ggml_type, pt.shape)
        w.write()
        paths.append(pp)
    return paths


def import_ik(rows, t, shape, device="cpu"):
    """Packed ik_llama rows -> (import type, its packed rows), via the fp32 values."""
    from ..gguf import dequantize, quantize
    from ..gguf.ik_quants import import_type

    tt = import_type(t)
    x = torch.from_numpy(dequantize(np.asarray(rows), t, (int(np.prod(shape[:-1])), shape[-1])))
    q = quantize(x.to(device), tt)
    return tt, q.reshape(x.shape[0], -1)


def tensors_from_gguf(g, device: str | torch.device = "cpu", names: set[str] | None = None) -> dict[str, PackedTensor]:
    """Wrap every tensor of a parsed GGUF as a PackedTensor (upload to ``device``)."""
    out = {}
    for name, ti in g.tensors.items():
        if names is not None and name not in names:
            continue
        shape = ti.torch_shape
        rows = ti.rows()
        if ti.ggml_type in IK_TYPES:  # ik_llama row-scaled types: requantize to a streamed type
            tt, data = import_ik(rows, ti.ggml_type, shape, device)
            out[name] = PackedTensor(name, tt, shape, data)
            continue
        if ti.ggml_type in (GGMLType.TQ1_0, GGMLType.TQ2_0):  # ternary: lossless repack to Q4_0
            from ..gguf.ternary import to_q4_0

            q4 = to_q4_0(np.asarray(rows), ti.ggml_type == GGMLType.TQ1_0).reshape(rows.shape[0], -1)
            out[name] = PackedTensor(name, GGMLType.Q4_0, shape, torch.from_numpy(q4).to(device))
            continue
        data = torch.from_numpy(np.array(rows, copy=True)).to(device)
        out[name] = PackedTensor(name, ti.ggml_type, shape, data)
    return out
