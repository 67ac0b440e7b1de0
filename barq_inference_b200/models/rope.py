"""RoPE frequency tables: plain, linear, NTK-aware and YaRN scaling.

The reference's core RoPE uses ``theta = base * exp2(2i/d)`` (``barq_core/src/rope.rs:23``), which is
not ``base^(2i/d)``, and its YaRN is a position-piecewise heuristic (``advanced/src/rope_scaling.rs``).
These tables follow the published definitions instead:

* linear: positions divided by ``factor``;
* NTK-aware: ``base' = base * factor^(d/(d-2))``;
* per-dimension frequency factors (GGUF ``rope_freqs.weight``, Llama-3.1 style): each inverse
  frequency divided by its factor, in any mode;
* LongRoPE (Ding et al. 2024, the Phi-3 scheme): long or short per-dimension factors as above, and
  the attention factor ``sqrt(1 + ln(s) / ln(orig_ctx))`` (s = context / original context) or the
  GGUF ``rope.scaling.attn_factor`` folded into cos/sin;
* YaRN (Peng et al. 2023): per-dimension ramp between interpolated and extrapolated angles over the
  correction range given by ``beta_fast``/``beta_slow``, and the attention temperature
  ``mscale = 1 + 0.1 ln(factor)`` folded into cos/sin.

Tables are precomputed once per model as float32 ``[max_pos, rot_dim/2]`` cos and sin; the fused
RMSNorm+RoPE kernels read them, so every scaling mode costs the same on the device.
"""
from __future__ import annotations

import math

import torch

from .config import ModelConfig


def _yarn_corr_dim(n_dims: int, n_ctx_orig: int, n_rot: float, base: float) -> float:
    return n_dims * math.log(n_ctx_orig / (n_rot * 2 * math.pi)) / (2 * math.log(base))


def rope_angles(cfg: ModelConfig, max_pos: int) -> tuple[torch.Tensor, float]:
    """Return (theta [max_pos, rot/2] float64, mscale) for the model's RoPE mode."""
    d = cfg.rot_dim
    base = cfg.rope_theta
    i = torch.arange(0, d // 2, dtype=torch.float64)
    pos = torch.arange(max_pos, dtype=torch.float64)[:, None]
    mscale = 1.0
    if cfg.rope_scaling == "ntk" and cfg.rope_factor > 1:
        base = base * cfg.rope_factor ** (d / (d - 2))
    inv = base ** (-2.0 * i / d)
    if cfg.rope_freq_factors:
        inv = inv / torch.tensor(cfg.rope_freq_factors, dtype=torch.float64)
    theta_ext = pos * inv
    if cfg.rope_scaling == "longrope":
        orig = cfg.rope_orig_ctx or cfg.max_ctx
        s = cfg.max_ctx / orig
        if cfg.rope_attn_factor > 0:
            mscale = cfg.rope_attn_factor
        elif s > 1:
            mscale = math.sqrt(1.0 + math.log(s) / math.log(orig))
        return theta_ext, mscale
    if cfg.rope_scaling == "linear" and cfg.rope_factor > 1:
        return theta_ext / cfg.rope_factor, mscale
    if cfg.rope_scaling == "yarn" and cfg.rope_factor > 1:
        fs = 1.0 / cfg.rope_factor
        n_orig = cfg.rope_orig_ctx or cfg.max_ctx
        low = max(0.0, math.floor(_yarn_corr_dim(d, n_orig, cfg.yarn_beta_fast, base)))
        high = min(d - 1.0, math.ceil(_yarn_corr_dim(d, n_orig, cfg.yarn_beta_slow, base)))
        y = (i - low) / max(0.001, high - low)
        ramp_mix = 1.0 - y.clamp(0.0, 1.0)  # 1 -> pure extrapolation (high-frequency dims)
        theta_int = theta_ext * fs
        theta = theta_int * (1 - ramp_mix) + theta_ext * ramp_mix
        mscale = 1.0 + 0.1 * math.log(1.0 / fs)
        if cfg.is_mla:
            # DeepSeek-V2 folds the YaRN temperature into the softmax scale instead (see attn_scale).
            mscale = 1.0
        return theta, mscale
    return theta_ext, mscale


def rope_cos_sin(cfg: ModelConfig, max_pos: int, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    theta, ms = rope_angles(cfg, max_pos)
    return (torch.cos(theta) * ms).float().to(device), (torch.sin(theta) * ms).float().to(device)


def attn_scale(cfg: ModelConfig) -> float:
    """Softmax scale 1/sqrt(d_k), with DeepSeek-V2's YaRN mscale^2 correction for MLA."""
    if cfg.is_mla:
        s = 1.0 / math.sqrt(cfg.qk_nope_dim + cfg.qk_rope_dim)
        if cfg.rope_scaling == "yarn" and cfg.rope_factor > 1:
            m = 1.0 + cfg.yarn_log_mul * math.log(cfg.rope_factor)
            s *= m * m
        return s
    return 1.0 / math.sqrt(cfg.head_dim)


def apply_rope_ref(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, neox: bool) -> torch.Tensor:
    """x: [T, H, rot]; cos/sin: [T, rot/2].  Reference (fp32) rotation for either pairing."""
    c = cos[:, None, :]
    s = sin[:, None, :]
    if neox:
        h = x.shape[-1] // 2
        x0, x1 = x[..., :h], x[..., h:]
        return torch.cat([x0 * c - x1 * s, x0 * s + x1 * c], -1)
    x0, x1 = x[..., 0::2], x[..., 1::2]
    out = torch.empty_like(x)
    out[..., 0::2] = x0 * c - x1 * s
    out[..., 1::2] = x0 * s + x1 * c
    return out
