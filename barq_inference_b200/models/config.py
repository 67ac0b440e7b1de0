"""Model hyper-parameters extracted from GGUF metadata, plus the benchmark presets.

Parity: ``ModelHParams`` / ``extract_hparams`` (``models/src/loader.rs:17-55,240-444``) and the
architecture registry (``models/src/arch.rs:7-151``, ``arch_registry.rs:343-434``).  The reference
reads only ``{llama,qwen,qwen2,qwen3,deepseek}.*`` keys and misses the RMS epsilon; here every
key the forward pass needs is read (rms eps, rope scaling, sliding window, experts, MLA ranks).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field, replace
from typing import Any

# GGUF architecture strings -> model family implemented in ``models/``.
ARCH_FAMILY = {
    "llama": "llama",
    "mistral": "llama",
    "mixtral": "llama",  # llama.cpp writes Mixtral as arch "llama" with expert_count > 0
    "qwen": "llama",
    "qwen2": "llama",
    "qwen2moe": "llama",
    "qwen3": "llama",
    "qwen3moe": "llama",
    "deepseek": "llama",
    "deepseek2": "deepseek2",
    "llava": "llama",  # the language half of a LLaVA checkpoint
    "qwen2vl": "llama",  # the language half of a Qwen2-VL checkpoint (qwen2 layers)
}

# RoPE pairing: ggml "normal" (adjacent pairs) vs NeoX (split halves).
NEOX_ARCHES = {"qwen", "qwen2", "qwen2moe", "qwen3", "qwen3moe", "qwen2vl"}


@dataclass
class ModelConfig:
    arch: str = "llama"
    n_layers: int = 2
    hidden: int = 256
    n_heads: int = 4
    n_kv_heads: int = 2
    head_dim: int = 64
    ffn: int = 688
    vocab: int = 32000
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_dim: int = 0  # 0 -> head_dim
    rope_neox: bool = False
    rope_scaling: str = "none"  # none | linear | yarn | ntk
    rope_factor: float = 1.0
    rope_orig_ctx: int = 0
    yarn_beta_fast: float = 32.0
    yarn_beta_slow: float = 1.0
    yarn_log_mul: float = 0.0  # deepseek2 rope.scaling.yarn_log_multiplier
    # per-dimension divisors of the RoPE inverse frequencies (rot_dim/2 values): the GGUF
    # ``rope_freqs.weight`` tensor (Llama-3.1-style scaling) or LongRoPE's long/short factor list
    rope_freq_factors: tuple = ()
    rope_attn_factor: float = 0.0  # cos/sin magnitude (LongRoPE attention factor); 0 -> derived
    max_ctx: int = 4096
    sliding_window: int = 0
    qkv_bias: bool = False
    qk_norm: bool = False
    tied_embeddings: bool = False
    # MoE
    n_experts: int = 0
    n_experts_used: int = 0
    expert_ffn: int = 0
    n_shared_experts: int = 0
    shared_expert_ffn: int = 0
    n_dense_layers: int = 0  # leading dense blocks (deepseek2)
    expert_gating: str = "softmax"  # softmax | sigmoid
    expert_weights_norm: bool = False
    expert_weights_scale: float = 1.0
    n_expert_groups: int = 1
    n_group_used: int = 1
    # MLA (deepseek2)
    q_lora_rank: int = 0
    kv_lora_rank: int = 0
    qk_nope_dim: int = 0
    qk_rope_dim: int = 0
    v_head_dim: int = 0
    # tokenizer
    bos_id: int = 1
    eos_ids: tuple[int, ...] = (2,)
    extra: dict[str, Any] = field(default_factory=dict)

    @property
    def is_moe(self) -> bool:
        return self.n_experts > 0

    @property
    def is_mla(self) -> bool:
        return self.kv_lora_rank > 0

    @property
    def rot_dim(self) -> int:
        if self.is_mla:
            return self.qk_rope_dim
        return self.rope_dim or self.head_dim

    @property
    def q_dim(self) -> int:
        return self.n_heads * self.head_dim

    @property
    def kv_dim(self) -> int:
        return self.n_kv_heads * self.head_dim

    def layer_is_moe(self, i: int) -> bool:
        return self.is_moe and i >= self.n_dense_layers

    def to_dict(self) -> dict:
        return asdict(self)

    def n_params(self) -> int:
        h = self.hidden
        attn = h * self.q_dim + 2 * h * self.kv_dim + self.q_dim * h
        if self.is_mla:
            qh = self.qk_nope_dim + self.qk_rope_dim
            attn = h * self.n_heads * qh + h * (self.kv_lora_rank + self.qk_rope_dim)
            attn += self.kv_lora_rank * self.n_heads * (self.qk_nope_dim + self.v_head_dim) + self.n_heads * self.v_head_dim * h
        total = 2 * self.vocab * h
        for i in range(self.n_layers):
            total += attn
            if self.layer_is_moe(i):
                total += self.n_experts * 3 * h * self.expert_ffn + h * self.n_experts
                total += self.n_shared_experts * 3 * h * (self.shared_expert_ffn or self.expert_ffn)
            else:
                total += 3 * h * self.ffn
        return total


def _g(md: dict, arch: str, key: str, default=None):
    for k in (f"{arch}.{key}", f"llama.{key}"):
        if k in md:
            return md[k]
    return default


def config_from_gguf(md: dict[str, Any], tensor_names: set[str] | None = None) -> ModelConfig:
    arch = str(md.get("general.architecture", "llama"))
    hidden = int(_g(md, arch, "embedding_length", 4096))
    n_heads = int(_g(md, arch, "attention.head_count", 32))
    kvh = _g(md, arch, "attention.head_count_kv", n_heads)
    if isinstance(kvh, (list, tuple)):
        kvh = kvh[0]
    head_dim = int(_g(md, arch, "attention.key_length", hidden // n_heads))
    ffn = _g(md, arch, "feed_forward_length", 4 * hidden)
    if isinstance(ffn, (list, tuple)):
        ffn = max(ffn)
    toks = md.get("tokenizer.ggml.tokens")
    vocab = int(_g(md, arch, "vocab_size", len(toks) if toks is not None else 32000))
    scaling = str(_g(md, arch, "rope.scaling.type", "none") or "none")
    cfg = ModelConfig(
        arch=arch,
        n_layers=int(_g(md, arch, "block_count", 32)),
        hidden=hidden,
        n_heads=n_heads,
        n_kv_heads=int(kvh),
        head_dim=head_dim,
        ffn=int(ffn),
        vocab=vocab,
        rms_eps=float(_g(md, arch, "attention.layer_norm_rms_epsilon", 1e-5)),
        rope_theta=float(_g(md, arch, "rope.freq_base", 10000.0)),
        rope_dim=int(_g(md, arch, "rope.dimension_count", 0) or 0),
        rope_neox=arch in NEOX_ARCHES,
        rope_scaling=scaling,
        rope_factor=float(_g(md, arch, "rope.scaling.factor", 1.0) or 1.0),
        rope_orig_ctx=int(_g(md, arch, "rope.scaling.original_context_length", 0) or 0),
        yarn_log_mul=float(_g(md, arch, "rope.scaling.yarn_log_multiplier", 0.0) or 0.0),
        rope_attn_factor=float(_g(md, arch, "rope.scaling.attn_factor", 0.0) or 0.0),
        max_ctx=int(_g(md, arch, "context_length", 4096)),
        sliding_window=int(_g(md, arch, "attention.sliding_window", 0) or 0),
        n_experts=int(_g(md, arch, "expert_count", 0) or 0),
        n_experts_used=int(_g(md, arch, "expert_used_count", 0) or 0),
        expert_ffn=int(_g(md, arch, "expert_feed_forward_length", 0) or 0),
        n_shared_experts=int(_g(md, arch, "expert_shared_count", 0) or 0),
        shared_expert_ffn=int(_g(md, arch, "expert_shared_feed_forward_length", 0) or 0),
        n_dense_layers=int(_g(md, arch, "leading_dense_block_count", 0) or 0),
        expert_weights_norm=bool(_g(md, arch, "expert_weights_norm", False)),
        expert_weights_scale=float(_g(md, arch, "expert_weights_scale", 1.0) or 1.0),
        expert_gating={1: "softmax", 2: "sigmoid"}.get(int(_g(md, arch, "expert_gating_func", 1) or 1), "softmax"),
        n_expert_groups=int(_g(md, arch, "expert_group_count", 1) or 1),
        n_group_used=int(_g(md, arch, "expert_group_used_count", 1) or 1),
        q_lora_rank=int(_g(md, arch, "attention.q_lora_rank", 0) or 0),
        kv_lora_rank=int(_g(md, arch, "attention.kv_lora_rank", 0) or 0),
        bos_id=int(md.get("tokenizer.ggml.bos_token_id", 1)),
    )
    eos = [int(md.get("tokenizer.ggml.eos_token_id", 2))]
    for k in ("tokenizer.ggml.eot_token_id", "tokenizer.ggml.eom_token_id"):
        if k in md:
            eos.append(int(md[k]))
    cfg.eos_ids = tuple(dict.fromkeys(eos))
    if cfg.is_mla:
        cfg.qk_rope_dim = int(_g(md, arch, "rope.dimension_count", 64) or 64)
        kl = int(_g(md, arch, "attention.key_length", 192))
        cfg.qk_nope_dim = kl - cfg.qk_rope_dim
        cfg.v_head_dim = int(_g(md, arch, "attention.value_length", 128))
        cfg.head_dim = kl
    if tensor_names is not None:
        cfg.qkv_bias = "blk.0.attn_q.bias" in tensor_names
        cfg.qk_norm = "blk.0.attn_q_norm.weight" in tensor_names
        cfg.tied_embeddings = "output.weight" not in tensor_names
    if arch in ("qwen2", "qwen2moe") and tensor_names is None:
        cfg.qkv_bias = True
    if arch in ("qwen3", "qwen3moe") and tensor_names is None:
        cfg.qk_norm = True
    return cfg


# --- presets for the benchmark configurations ---------------------------------------------

PRESETS: dict[str, ModelConfig] = {
    "tiny": ModelConfig(arch="llama", n_layers=2, hidden=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=688,
                        vocab=32000, rms_eps=1e-5, rope_theta=10000.0, max_ctx=512),
    # test-sized MoE (Mixtral-style: 4 experts, top-2, softmax gate)
    "tiny-moe": ModelConfig(arch="llama", n_layers=2, hidden=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=512,
                            vocab=4096, rms_eps=1e-5, rope_theta=10000.0, max_ctx=512, n_experts=4,
                            n_experts_used=2, expert_ffn=256),
    # test-sized DeepSeek-V2 (MLA with the real 16 heads / 512 latent / 64 rope; 1 dense + 1 MoE layer)
    "tiny-ds": ModelConfig(arch="deepseek2", n_layers=2, hidden=256, n_heads=16, n_kv_heads=16, head_dim=192,
                           ffn=512, vocab=4096, rms_eps=1e-6, rope_theta=10000.0, max_ctx=512, n_experts=4,
                           n_experts_used=2, expert_ffn=256, n_shared_experts=1, n_dense_layers=1,
                           expert_weights_norm=False, kv_lora_rank=512, qk_nope_dim=128, qk_rope_dim=64,
                           v_head_dim=128, bos_id=1, eos_ids=(2,)),
    "llama3-8b": ModelConfig(arch="llama", n_layers=32, hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128,
                             ffn=14336, vocab=128256, rms_eps=1e-5, rope_theta=500000.0, max_ctx=8192,
                             bos_id=128000, eos_ids=(128001, 128009)),
    "llama3-70b": ModelConfig(arch="llama", n_layers=80, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128,
                              ffn=28672, vocab=128256, rms_eps=1e-5, rope_theta=500000.0, max_ctx=32768,
                              rope_scaling="yarn", rope_factor=4.0, rope_orig_ctx=8192,
                              bos_id=128000, eos_ids=(128001, 128009)),
    "mixtral-8x7b": ModelConfig(arch="llama", n_layers=32, hidden=4096, n_heads=32, n_kv_heads=8, head_dim=128,
                                ffn=14336, vocab=32000, rms_eps=1e-5, rope_theta=1e6, max_ctx=32768,
                                sliding_window=4096, n_experts=8, n_experts_used=2, expert_ffn=14336),
    "deepseek-v2-lite": ModelConfig(arch="deepseek2", n_layers=27, hidden=2048, n_heads=16, n_kv_heads=16,
                                    head_dim=192, ffn=10944, vocab=102400, rms_eps=1e-6, rope_theta=10000.0,
                                    max_ctx=32768, rope_scaling="yarn", rope_factor=4.0, rope_orig_ctx=4096,
                                    yarn_log_mul=0.0707, n_experts=64, n_experts_used=6, expert_ffn=1408,
                                    n_shared_experts=2, n_dense_layers=1, expert_weights_norm=False,
                                    kv_lora_rank=512, qk_nope_dim=128, qk_rope_dim=64, v_head_dim=128,
                                    bos_id=100000, eos_ids=(100001,)),
}


def preset(name: str, **overrides) -> ModelConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; known: {sorted(PRESETS)}")
    return replace(PRESETS[name], **overrides)


def attach_rope_factors(cfg: ModelConfig, g) -> ModelConfig:
    """Reads per-dimension RoPE frequency factors from a parsed GGUF file into ``cfg``:
    ``rope_freqs.weight`` (Llama-3.1-style) or LongRoPE's ``rope_factors_long.weight`` /
    ``rope_factors_short.weight`` (long factors when the context exceeds the original one)."""
    import numpy as np

    def vec(name):
        t = g.tensors.get(name)
        if t is None:
            return None
        return tuple(float(x) for x in np.frombuffer(bytes(t.data), dtype=np.float32))

    ff = vec("rope_freqs.weight")
    long_f, short_f = vec("rope_factors_long.weight"), vec("rope_factors_short.weight")
    if long_f is not None or short_f is not None:
        cfg.rope_scaling = "longrope"
        orig = cfg.rope_orig_ctx or cfg.max_ctx
        use_long = long_f is not None and (cfg.max_ctx > orig or short_f is None)
        ff = long_f if use_long else short_f
    if ff is not None:
        if len(ff) != cfg.rot_dim // 2:
            raise ValueError(f"RoPE factor tensor has {len(ff)} values, expected rot_dim/2 = {cfg.rot_dim // 2}")
        cfg.rope_freq_factors = ff
    return cfg
