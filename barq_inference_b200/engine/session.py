"""KV session export / import: save the attention state of a prompt and resume from it later (another
process, another restart) without prefilling it again.

Parity: ``save_kv_state`` / ``restore_kv_state`` (``models/src/prompt_cache.rs:197-204``, in a module
the reference never compiles) and the prompt cache's purpose (``advanced/src/prompt_cache.rs``).

File format (``torch.save`` of plain tensors and scalars, loadable with ``weights_only=True``):
``{"format": "barq-kv-session", "version": 1, "arch", "n_layers", "n_kv_heads", "head_dim",
"tokens": int64 [n], "kv": {"k.<layer>": [n, Hkv, D], "v.<layer>": [n, Hkv, D]}}`` — or, for MLA
models on the CPU engine, ``"c.<layer>"`` / ``"kpe.<layer>"`` latent rows.  Rows are in position
order; their dtype is the cache's (fp32 from the CPU engine, fp16 / bf16 / fp8 from the GPU one)
and is converted to the importing cache's dtype.

* GPU ``Engine`` (prefix caching on, one rank): ``export_session`` reads the pages of the longest
  cached block-aligned prefix of the tokens (running a one-token generation first if nothing is
  cached); ``import_session`` writes the rows into fresh pages and donates them to the radix
  prefix cache, so any later request whose prompt starts with those tokens skips their prefill.
* ``CPUEngine``: ``export_session`` runs the prefill on the reference forward; ``import_session``
  stores the state, and a new request whose prompt extends it starts from a copy.
"""
from __future__ import annotations

import torch

FORMAT = "barq-kv-session"
VERSION = 1


def _meta(cfg) -> dict:
    return {"format": FORMAT, "version": VERSION, "arch": cfg.arch, "n_layers": cfg.n_layers,
            "n_kv_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim}


def save_session(state: dict, path: str) -> None:
    torch.save(state, path)


def load_session(path: str) -> dict:
    state = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(state, dict) or state.get("format") != FORMAT:
        raise ValueError(f"{path}: not a barq KV session file")
    if int(state.get("version", 0)) > VERSION:
        raise ValueError(f"{path}: session format version {state['version']} is newer than this build ({VERSION})")
    return state


def _check(engine, state: dict) -> None:
    cfg = engine.cfg
    for k in ("arch", "n_layers", "n_kv_heads", "head_dim"):
        if state[k] != getattr(cfg, k):
            raise ValueError(f"session {k}={state[k]!r} does not match the model ({getattr(cfg, k)!r})")


# ------------------------------------------------------------------ CPU engine
def _cpu_export(engine, tokens: list[int]) -> dict:
    cache: dict = {}
    with torch.no_grad():
        engine.model.forward(list(tokens), cache)
    kv = {f"{key[0]}.{key[1]}": t.contiguous().clone() for key, t in cache.items() if isinstance(key, tuple)}
    return {**_meta(engine.cfg), "tokens": torch.tensor(tokens, dtype=torch.int64), "kv": kv}


def _cpu_import(engine, state: dict) -> int:
    toks = [int(t) for t in state["tokens"].tolist()]
    cache: dict = {"pos": len(toks)}
    for name, t in state["kv"].items():
        kind, layer = name.rsplit(".", 1)
        cache[(kind, int(layer))] = t.float()
    engine.sessions.append((toks, cache))
    return len(toks)


# ------------------------------------------------------------------ GPU engine (paged KV)
def _paged_kv(engine):
    runner = engine.runner
    kv = getattr(runner, "kv", None)
    if getattr(engine.cfg, "is_mla", False) or not kv or kv[0][0].dim() != 4:
        raise NotImplementedError("KV sessions cover the paged K/V cache of MHA/GQA models")
    if getattr(engine.ecfg, "tp", 1) > 1 or getattr(engine.ecfg, "pp", 1) > 1:
        raise NotImplementedError("KV sessions are single-rank (tp = pp = 1)")
    if engine.prefix_cache is None:
        raise ValueError("KV sessions on the GPU engine need prefix caching (EngineConfig.prefix_caching=True)")
    return kv


def _scales(engine, layer: int):
    """(K scales, V scales) [num_blocks, Hkv, block_size] of a scaled fp8 cache, else None."""
    sc = getattr(engine.runner, "kv_scales", None)
    return sc[layer] if sc else None


def _bytes(t: torch.Tensor) -> torch.Tensor:
    """1-byte element types (fp8) viewed as uint8 for gathers and scatters."""
    return t.view(torch.uint8) if t.element_size() == 1 else t


def _gpu_export(engine, tokens: list[int]) -> dict:
    kv = _paged_kv(engine)
    blocks, n = engine.prefix_cache.match(list(tokens))
    if n == 0:
        from .sampling_params import SamplingParams

        engine.generate([list(tokens)], SamplingParams.greedy_params(max_tokens=1))
        blocks, n = engine.prefix_cache.match(list(tokens))
    if n == 0:
        raise ValueError("prompt shorter than one KV page: nothing to export")
    idx = torch.tensor(blocks, dtype=torch.long, device=kv[0][0].device)
    out = {}
    for i, (K, V) in enumerate(kv):
        # [nb, Hkv, bs, D] pages -> [nb * bs, Hkv, D] rows in position order
        for name, P in (("k", K), ("v", V)):
            pg = _bytes(P).index_select(0, idx).view(P.dtype)  # fp8 pages move as bytes
            out[f"{name}.{i}"] = pg.permute(0, 2, 1, 3).reshape(-1, pg.shape[1], pg.shape[3]).cpu()
        sc = _scales(engine, i)
        for name, S in (() if sc is None else (("ks", sc[0]), ("vs", sc[1]))):  # fp8: per-row scales
            out[f"{name}.{i}"] = S.index_select(0, idx).permute(0, 2, 1).reshape(-1, S.shape[1]).cpu()
    return {**_meta(engine.cfg), "tokens": torch.tensor(list(tokens)[:n], dtype=torch.int64), "kv": out}


def _gpu_import(engine, state: dict) -> int:
    kv = _paged_kv(engine)
    bs = engine.blocks.block_size
    toks = [int(t) for t in state["tokens"].tolist()]
    nb = len(toks) // bs
    if nb == 0:
        return 0
    if not engine.blocks.can_allocate(nb):
        engine.prefix_cache.evict(nb - engine.blocks.n_free)
    blocks = engine.blocks.allocate(nb)
    idx = torch.tensor(blocks, dtype=torch.long, device=kv[0][0].device)
    for i, (K, V) in enumerate(kv):
        for name, P in (("k", K), ("v", V)):
            rows = state["kv"][f"{name}.{i}"][: nb * bs]
            pg = rows.to(P.dtype).reshape(nb, bs, rows.shape[1], rows.shape[2]).permute(0, 2, 1, 3).contiguous()
            _bytes(P).index_copy_(0, idx, _bytes(pg).to(P.device))
        sc = _scales(engine, i)
        for name, S in (() if sc is None else (("ks", sc[0]), ("vs", sc[1]))):
            rows = state["kv"].get(f"{name}.{i}")
            if rows is None:
                raise ValueError("the session has no per-row scales for this fp8 KV cache")
            pg = rows[: nb * bs].to(S.dtype).reshape(nb, bs, S.shape[1]).permute(0, 2, 1).contiguous()
            S.index_copy_(0, idx, pg.to(S.device))
    engine.prefix_cache.insert(toks[: nb * bs], blocks)  # the cache takes its own reference
    engine.blocks.release(blocks)
    return nb * bs


# ------------------------------------------------------------------ public
def export_session(engine, tokens: list[int], path: str | None = None) -> dict:
    """The KV state of ``tokens`` (GPU engine: of their longest cached block-aligned prefix); written
    to ``path`` when given."""
    state = _cpu_export(engine, tokens) if hasattr(engine, "sessions") else _gpu_export(engine, tokens)
    if path is not None:
        save_session(state, path)
    return state


def import_session(engine, state_or_path) -> int:
    """Makes a saved state available to later requests; returns the number of tokens whose prefill
    those requests will skip."""
    state = load_session(state_or_path) if isinstance(state_or_path, str) else state_or_path
    _check(engine, state)
    return _cpu_import(engine, state) if hasattr(engine, "sessions") else _gpu_import(engine, state)
