"""fp32 reference forward pass (the correctness oracle for every model family).

Restates the reference's dense decoder math (``models/src/transformer.rs:81-498``: embedding
gather, pre-norm RMSNorm, Q/K/V projections with optional bias, RoPE, causal GQA attention,
SwiGLU FFN, final norm, output head with tied-embedding fallback) from dequantized f32 weights,
and adds what the reference never executes: sliding-window masks, Qwen3 QK-norm, top-k MoE with
SER, and DeepSeek-V2 MLA with shared experts.  It is deliberately simple and exact; the engine's
CUDA path is checked against it.
"""
from __future__ import annotations


import numpy as np
import torch
import torch.nn.functional as F

from ..gguf import dequantize
from .config import ModelConfig
from .rope import apply_rope_ref, attn_scale, rope_cos_sin
from .weights import PackedTensor


def dequant_tensor(pt: PackedTensor) -> torch.Tensor:
    arr = dequantize(pt.data.cpu().numpy(), pt.ggml_type, pt.shape)
    return torch.from_numpy(np.ascontiguousarray(arr))


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w


def moe_route(logits: torch.Tensor, cfg: ModelConfig, ser_threshold: float = 0.0):
    """Return (topk ids [T,k], weights [T,k]).  Softmax gate, top-k, optional renorm and SER."""
    if cfg.expert_gating == "sigmoid":
        probs = torch.sigmoid(logits)
    else:
        probs = torch.softmax(logits, -1)
    w, ids = torch.topk(probs, cfg.n_experts_used, dim=-1)
    if cfg.arch != "deepseek2" or cfg.expert_weights_norm:
        w = w / w.sum(-1, keepdim=True)
    if ser_threshold > 0:
        keep = w >= ser_threshold
        keep[:, 0] = True
        w = torch.where(keep, w, torch.zeros_like(w))
        w = w / w.sum(-1, keepdim=True)
    return ids, w * cfg.expert_weights_scale


class ReferenceModel:
    def __init__(self, cfg: ModelConfig, tensors: dict[str, PackedTensor], ser_threshold: float = 0.0):
        self.cfg = cfg
        self.ser = ser_threshold
        self.w = {k: dequant_tensor(v) for k, v in tensors.items()}
        self.cos, self.sin = rope_cos_sin(cfg, cfg.max_ctx)
        self.scale = attn_scale(cfg)

    def to(self, device) -> "ReferenceModel":
        """Move the dequantized weights and RoPE tables (e.g. to a GPU for context-parallel prefill)."""
        self.w = {k: v.to(device) for k, v in self.w.items()}
        self.cos, self.sin = self.cos.to(device), self.sin.to(device)
        return self

    def _attn(self, q, k, v, T0: int):
        """q: [T,H,d], k/v: [S,Hkv,d] with the last T rows new; causal (+SWA) mask."""
        cfg = self.cfg
        T, H, _ = q.shape
        S = k.shape[0]
        rep = H // k.shape[1]
        k = k.repeat_interleave(rep, 1)
        v = v.repeat_interleave(rep, 1)
        s = torch.einsum("thd,shd->hts", q, k) * self.scale
        qpos = torch.arange(T0, T0 + T)[:, None]
        kpos = torch.arange(S)[None, :]
        mask = kpos > qpos
        if cfg.sliding_window:
            mask |= kpos <= qpos - cfg.sliding_window
        s = s.masked_fill(mask[None], float("-inf"))
        p = torch.softmax(s, -1)
        return torch.einsum("hts,shd->thd", p, v)

    def _ffn(self, x, p):
        w = self.w
        g = x @ w[p + "ffn_gate.weight"].T
        u = x @ w[p + "ffn_up.weight"].T
        return (F.silu(g) * u) @ w[p + "ffn_down.weight"].T

    def _moe(self, x, p):
        cfg, w = self.cfg, self.w
        logits = x @ w[p + "ffn_gate_inp.weight"].T
        ids, wt = moe_route(logits, cfg, self.ser)
        load = getattr(self, "expert_load", None)
        if load is not None:
            load.add(int(p.split(".")[1]), torch.bincount(ids.reshape(-1), minlength=cfg.n_experts))
        out = torch.zeros_like(x)
        G, U, D = w[p + "ffn_gate_exps.weight"], w[p + "ffn_up_exps.weight"], w[p + "ffn_down_exps.weight"]
        for t in range(x.shape[0]):
            for j in range(ids.shape[1]):
                if wt[t, j] == 0:
                    continue
                e = int(ids[t, j])
                h = F.silu(x[t] @ G[e].T) * (x[t] @ U[e].T)
                out[t] += wt[t, j] * (h @ D[e].T)
        if cfg.n_shared_experts:
            g = x @ w[p + "ffn_gate_shexp.weight"].T
            u = x @ w[p + "ffn_up_shexp.weight"].T
            out += (F.silu(g) * u) @ w[p + "ffn_down_shexp.weight"].T
        return out

    def forward(self, ids: list[int] | torch.Tensor, cache: dict | None = None,
                embeds: tuple[int, torch.Tensor] | None = None, hidden: bool = False) -> torch.Tensor:
        """Logits for every position of ``ids``.  ``cache`` (dict) carries K/V across calls.
        ``embeds`` = (first row, [n, hidden]) replaces those rows' token embeddings."""
        cfg, w = self.cfg, self.w
        ids = torch.as_tensor(ids, dtype=torch.long)
        if cache is None:
            cache = {}
        T0 = cache.get("pos", 0)
        T = ids.numel()
        x = w["token_embd.weight"][ids]
        if embeds is not None:
            x = x.clone()
            x[embeds[0]: embeds[0] + embeds[1].shape[0]] = embeds[1].to(x.dtype).cpu()
        cos, sin = self.cos[T0 : T0 + T], self.sin[T0 : T0 + T]
        for i in range(cfg.n_layers):
            p = f"blk.{i}."
            hN = rms_norm(x, w[p + "attn_norm.weight"], cfg.rms_eps)
            if cfg.is_mla:
                a = self._mla(hN, p, i, cache, cos, sin, T0)
            else:
                q = hN @ w[p + "attn_q.weight"].T
                k = hN @ w[p + "attn_k.weight"].T
                v = hN @ w[p + "attn_v.weight"].T
                if cfg.qkv_bias:
                    q = q + w[p + "attn_q.bias"]
                    k = k + w[p + "attn_k.bias"]
                    v = v + w[p + "attn_v.bias"]
                q = q.view(T, cfg.n_heads, cfg.head_dim)
                k = k.view(T, cfg.n_kv_heads, cfg.head_dim)
                v = v.view(T, cfg.n_kv_heads, cfg.head_dim)
                if cfg.qk_norm:
                    q = rms_norm(q, w[p + "attn_q_norm.weight"], cfg.rms_eps)
                    k = rms_norm(k, w[p + "attn_k_norm.weight"], cfg.rms_eps)
                r = cfg.rot_dim
                q = torch.cat([apply_rope_ref(q[..., :r], cos, sin, cfg.rope_neox), q[..., r:]], -1)
                k = torch.cat([apply_rope_ref(k[..., :r], cos, sin, cfg.rope_neox), k[..., r:]], -1)
                kc = torch.cat([cache.get(("k", i), k[:0]), k], 0)
                vc = torch.cat([cache.get(("v", i), v[:0]), v], 0)
                cache[("k", i)], cache[("v", i)] = kc, vc
                o = self._attn(q, kc, vc, T0).reshape(T, -1)
                a = o @ w[p + "attn_output.weight"].T
            x = x + a
            hN = rms_norm(x, w[p + "ffn_norm.weight"], cfg.rms_eps)
            x = x + (self._moe(hN, p) if cfg.layer_is_moe(i) else self._ffn(hN, p))
        x = rms_norm(x, w["output_norm.weight"], cfg.rms_eps)
        cache["pos"] = T0 + T
        if hidden:  # final-norm hidden states instead of logits (embeddings)
            return x
        head = w.get("output.weight", w["token_embd.weight"])
        return x @ head.T

    def _mla(self, x, p, i, cache, cos, sin, T0):
        cfg, w = self.cfg, self.w
        T = x.shape[0]
        H, dn, dr, dv, L = cfg.n_heads, cfg.qk_nope_dim, cfg.qk_rope_dim, cfg.v_head_dim, cfg.kv_lora_rank
        if cfg.q_lora_rank:
            qa = rms_norm(x @ w[p + "attn_q_a.weight"].T, w[p + "attn_q_a_norm.weight"], cfg.rms_eps)
            q = qa @ w[p + "attn_q_b.weight"].T
        else:
            q = x @ w[p + "attn_q.weight"].T
        q = q.view(T, H, dn + dr)
        q_nope, q_pe = q[..., :dn], q[..., dn:]
        kva = x @ w[p + "attn_kv_a_mqa.weight"].T
        c = rms_norm(kva[:, :L], w[p + "attn_kv_a_norm.weight"], cfg.rms_eps)
        k_pe = kva[:, L:].view(T, 1, dr)
        q_pe = apply_rope_ref(q_pe, cos, sin, cfg.rope_neox)
        k_pe = apply_rope_ref(k_pe, cos, sin, cfg.rope_neox)
        cc = torch.cat([cache.get(("c", i), c[:0]), c], 0)
        kp = torch.cat([cache.get(("kpe", i), k_pe[:0]), k_pe], 0)
        cache[("c", i)], cache[("kpe", i)] = cc, kp
        kv = (cc @ w[p + "attn_kv_b.weight"].T).view(cc.shape[0], H, dn + dv)
        k = torch.cat([kv[..., :dn], kp.expand(-1, H, -1)], -1)
        v = kv[..., dn:]
        qf = torch.cat([q_nope, q_pe], -1)
        o = self._attn(qf, k, v, T0).reshape(T, H * dv)
        return o @ w[p + "attn_output.weight"].T

    @torch.no_grad()
    def greedy(self, prompt: list[int], n: int) -> tuple[list[int], list[torch.Tensor]]:
        cache: dict = {}
        logits = self.forward(prompt, cache)[-1]
        out, all_logits = [], []
        for _ in range(n):
            all_logits.append(logits)
            t = int(torch.argmax(logits))
            out.append(t)
            logits = self.forward([t], cache)[-1]
        return out, all_logits
