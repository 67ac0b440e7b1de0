"""Context parallelism: ring-attention prefill for prompts too long for one GPU's attention pass.

Parity: none in the reference — its long-context support is paged KV, RoPE scaling and the ``--mla``
context multiplier (``advanced/src/paged_attention.rs``, ``advanced/src/rope_scaling.rs``,
``advanced/src/flash_mla.rs:89-117``); there is no context parallelism, ring attention or Ulysses.

Layout: the prompt's T positions are cut into ``2 * world`` equal chunks and rank r holds chunks r
and ``2*world-1-r`` ("zigzag"), so under the causal mask every rank has the same amount of work.
Each rank keeps its own queries; the K/V shards travel around the ring, one hop per round, while
the current shard is being used: round i posts the send of the shard in hand to the next rank and
the receive of the previous rank's shard, computes with the shard in hand, then waits.  Partial
results are merged with the log-sum-exp (online softmax) rule, so the output equals full causal
attention.  On GPUs the hops are NCCL send/recv over NVLink (``torch.distributed`` P2P) and the
block math is batched matmuls; on CPU the same code runs over ``gloo`` (tests).

Functions: ``zigzag_indices`` (which positions a rank holds), ``ring_attention`` (the op),
``gather_zigzag`` (reassemble a per-rank tensor in position order, e.g. to hand the K/V of a
context-parallel prefill to a single-GPU decode engine).
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist


def zigzag_indices(T: int, world: int, rank: int) -> torch.Tensor:
    """Positions held by ``rank``: chunks ``rank`` and ``2*world-1-rank`` of ``2*world`` equal chunks."""
    if T % (2 * world):
        raise ValueError(f"sequence length {T} must be a multiple of 2 * world = {2 * world}")
    c = T // (2 * world)
    a, b = rank, 2 * world - 1 - rank
    return torch.cat([torch.arange(a * c, (a + 1) * c), torch.arange(b * c, (b + 1) * c)])


def _block_attn(q, k, v, qpos, kpos, scale, causal: bool, window: int):
    """Attention of q [Hq, Tq, D] against one K/V shard [Hkv, Tk, D] (GQA: Hq multiple of Hkv).
    Returns (out [Hq, Tq, D] normalized within the shard, lse [Hq, Tq]); rows with no visible key
    get lse = -inf and out = 0."""
    Hq, Hkv = q.shape[0], k.shape[0]
    g = Hq // Hkv
    qf = q.float().reshape(Hkv, g * q.shape[1], q.shape[2])
    s = torch.bmm(qf, k.float().transpose(1, 2)).reshape(Hq, q.shape[1], k.shape[1]) * scale
    mask = None
    if causal:
        mask = kpos[None, :] > qpos[:, None]
    if window > 0:
        w = kpos[None, :] <= qpos[:, None] - window
        mask = w if mask is None else (mask | w)
    if mask is not None:
        s = s.masked_fill(mask[None], float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse.clamp_min(-1e30)[..., None])
    p = torch.nan_to_num(p, nan=0.0)
    out = torch.bmm(p.reshape(Hkv, g * q.shape[1], k.shape[1]), v.float()).reshape(Hq, q.shape[1], v.shape[2])
    return out, lse


def _merge(out, lse, o2, l2):
    """Log-sum-exp merge of two partial attention results over disjoint key sets."""
    m = torch.maximum(lse, l2)
    m_safe = torch.where(torch.isfinite(m), m, torch.zeros_like(m))
    a = torch.exp(lse - m_safe)
    b = torch.exp(l2 - m_safe)
    den = a + b
    live = den > 0
    new = torch.where(live[..., None], (out * a[..., None] + o2 * b[..., None]) / den.clamp_min(1e-30)[..., None], out)
    new_lse = torch.where(live, m_safe + torch.log(den.clamp_min(1e-30)), torch.full_like(den, float("-inf")))
    return new, new_lse


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, positions: torch.Tensor,
                   scale: float | None = None, causal: bool = True, window: int = 0, group=None):
    """Context-parallel attention.  This rank holds queries and keys/values of the positions
    ``positions`` (any set, e.g. ``zigzag_indices``): ``q`` [Hq, n, D], ``k``/``v`` [Hkv, n, D].
    Every rank must hold the same number of positions.  Returns (out [Hq, n, D] in q's dtype,
    lse [Hq, n] fp32).  With one rank this is plain attention over the local positions."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    positions = positions.to(q.device)
    out = torch.zeros(q.shape[0], q.shape[1], v.shape[2], dtype=torch.float32, device=q.device)
    lse = torch.full(q.shape[:2], float("-inf"), dtype=torch.float32, device=q.device)
    # the travelling shard: K, V and their positions packed in one fp32 buffer so each hop is one
    # send (positions are exact in fp32 below 2**24)
    D, Dv = k.shape[2], v.shape[2]
    cur = torch.cat([k.float().reshape(-1), v.float().reshape(-1), positions.float()])
    nxt = torch.empty_like(cur) if world > 1 else None
    send_to, recv_from = (rank + 1) % world, (rank - 1) % world
    nk = k.numel()
    for i in range(world):
        reqs = []
        if i + 1 < world:
            gs = dist.get_global_rank(group, send_to) if group is not None else send_to
            gr = dist.get_global_rank(group, recv_from) if group is not None else recv_from
            ops = [dist.P2POp(dist.isend, cur, gs, group), dist.P2POp(dist.irecv, nxt, gr, group)]
            reqs = dist.batch_isend_irecv(ops)
        ks = cur[:nk].view(k.shape[0], -1, D)
        vs = cur[nk: nk + v.numel()].view(v.shape[0], -1, Dv)
        kp = cur[nk + v.numel():].round().long()
        o2, l2 = _block_attn(q, ks, vs, positions, kp, scale, causal, window)
        out, lse = _merge(out, lse, o2, l2)
        for r in reqs:
            r.wait()
        if i + 1 < world:
            cur, nxt = nxt, cur
    return out.to(q.dtype), lse


def gather_zigzag(x: torch.Tensor, T: int, dim: int = 1, group=None) -> torch.Tensor:
    """All-gather a per-rank tensor whose ``dim`` holds this rank's ``zigzag_indices`` and return
    it with ``dim`` in position order (length T)."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if world == 1:
        return x
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous(), group=group)
    full_shape = list(x.shape)
    full_shape[dim] = T
    outp = torch.empty(full_shape, dtype=x.dtype, device=x.device)
    for r, part in enumerate(parts):
        outp.index_copy_(dim, zigzag_indices(T, world, r).to(x.device), part)
    return outp


def cp_prefill(model, prompt: list[int], group=None):
    """Context-parallel prefill of a dense (non-MLA) decoder given as a ``ReferenceModel``: each rank
    runs every layer on its zigzag share of the prompt, attention is ``ring_attention``, and the K/V
    of every layer is gathered in position order into the returned cache, so decoding continues
    with ``model.forward([tok], cache)`` on any rank.  Returns (logits of the last prompt position,
    cache).  The prompt length must be a multiple of ``2 * world``."""
    from ..models.reference import rms_norm
    from ..models.rope import apply_rope_ref

    cfg, w = model.cfg, model.w
    if cfg.is_mla:
        raise NotImplementedError("context-parallel prefill covers MHA/GQA decoders")
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    T = len(prompt)
    dev = w["token_embd.weight"].device  # CPU, or a GPU after ``model.to(...)`` (NCCL ring)
    idx = zigzag_indices(T, world, rank).to(dev)
    ids = torch.as_tensor(prompt, dtype=torch.long, device=dev)[idx]
    n = ids.numel()
    x = w["token_embd.weight"][ids]
    cos, sin = model.cos[idx], model.sin[idx]
    cache: dict = {}
    for i in range(cfg.n_layers):
        p = f"blk.{i}."
        hN = rms_norm(x, w[p + "attn_norm.weight"], cfg.rms_eps)
        q, k, v = hN @ w[p + "attn_q.weight"].T, hN @ w[p + "attn_k.weight"].T, hN @ w[p + "attn_v.weight"].T
        if cfg.qkv_bias:
            q, k, v = q + w[p + "attn_q.bias"], k + w[p + "attn_k.bias"], v + w[p + "attn_v.bias"]
        q = q.view(n, cfg.n_heads, cfg.head_dim)
        k = k.view(n, cfg.n_kv_heads, cfg.head_dim)
        v = v.view(n, cfg.n_kv_heads, cfg.head_dim)
        if cfg.qk_norm:
            q = rms_norm(q, w[p + "attn_q_norm.weight"], cfg.rms_eps)
            k = rms_norm(k, w[p + "attn_k_norm.weight"], cfg.rms_eps)
        r = cfg.rot_dim
        q = torch.cat([apply_rope_ref(q[..., :r], cos, sin, cfg.rope_neox), q[..., r:]], -1)
        k = torch.cat([apply_rope_ref(k[..., :r], cos, sin, cfg.rope_neox), k[..., r:]], -1)
        o, _ = ring_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1), idx, scale=model.scale,
                              window=cfg.sliding_window, group=group)
        cache[("k", i)] = gather_zigzag(k, T, dim=0, group=group)
        cache[("v", i)] = gather_zigzag(v, T, dim=0, group=group)
        x = x + o.transpose(0, 1).reshape(n, -1) @ w[p + "attn_output.weight"].T
        hN = rms_norm(x, w[p + "ffn_norm.weight"], cfg.rms_eps)
        x = x + (model._moe(hN, p) if cfg.layer_is_moe(i) else model._ffn(hN, p))
    # position T-1 is the last row of rank 0's second chunk
    last = torch.zeros(cfg.hidden, dtype=x.dtype, device=dev)
    if rank == 0:
        last = x[-1].clone()
    if world > 1:
        dist.broadcast(last, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    h = rms_norm(last[None], w["output_norm.weight"], cfg.rms_eps)
    head = w.get("output.weight", w["token_embd.weight"])
    cache["pos"] = T
    return (h @ head.T)[0], cache
