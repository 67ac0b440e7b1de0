"""Context-parallel ring attention over gloo on CPU: zigzag shards of a causal (GQA, optionally
sliding-window) attention equal the full single-process attention."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from barq_inference_b200.parallel.cp import gather_zigzag, ring_attention, zigzag_indices


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _full(q, k, v, window):
    Hq, T, D = q.shape
    g = Hq // k.shape[0]
    kk, vv = k.repeat_interleave(g, 0), v.repeat_interleave(g, 0)
    s = q @ kk.transpose(1, 2) / D ** 0.5
    pos = torch.arange(T)
    mask = pos[None, :] > pos[:, None]
    if window:
        mask |= pos[None, :] <= pos[:, None] - window
    s = s.masked_fill(mask, float("-inf"))
    return torch.softmax(s, -1) @ vv


def _worker(rank, world, port, T, window, out_path):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    g = torch.Generator().manual_seed(0)
    q = torch.randn(8, T, 32, generator=g)
    k = torch.randn(2, T, 32, generator=g)
    v = torch.randn(2, T, 32, generator=g)
    idx = zigzag_indices(T, world, rank)
    out, lse = ring_attention(q[:, idx], k[:, idx], v[:, idx], idx, window=window)
    full = gather_zigzag(out, T, dim=1)
    if rank == 0:
        ref = _full(q, k, v, window)
        torch.save({"err": (full - ref).abs().max().item(), "finite": bool(torch.isfinite(lse).all())}, out_path)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,window", [(2, 0), (4, 0), (3, 20)])
def test_ring_attention_matches_full(world, window, tmp_path):
    T = 24 * world
    path = str(tmp_path / "r.pt")
    mp.spawn(_worker, args=(world, _free_port(), T, window, path), nprocs=world, join=True)
    r = torch.load(path)
    assert r["err"] < 1e-5, r
    assert r["finite"]


def test_zigzag_partition_and_single_rank():
    T, world = 32, 4
    allidx = torch.cat([zigzag_indices(T, world, r) for r in range(world)])
    assert sorted(allidx.tolist()) == list(range(T))
    # causal work is balanced: every rank's (query, visible key) pair count is equal
    work = [int((zigzag_indices(T, world, r) + 1).sum()) for r in range(world)]
    assert len(set(work)) == 1
    with pytest.raises(ValueError):
        zigzag_indices(30, 4, 0)
    q, k, v = torch.randn(4, 16, 8), torch.randn(4, 16, 8), torch.randn(4, 16, 8)
    out, _ = ring_attention(q, k, v, torch.arange(16))  # no process group: plain causal attention
    assert (out - _full(q, k, v, 0)).abs().max() < 1e-5


def _model_worker(rank, world, port, window, out_path):
    import dataclasses

    from barq_inference_b200.models import POLICIES, preset, random_tensors
    from barq_inference_b200.models.reference import ReferenceModel
    from barq_inference_b200.parallel.cp import cp_prefill

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    cfg = dataclasses.replace(preset("tiny", n_layers=2, vocab=500, max_ctx=256), sliding_window=window)
    model = ReferenceModel(cfg, random_tensors(cfg, POLICIES["tiny"], seed=3))
    prompt = torch.randint(0, cfg.vocab, (48,), generator=torch.Generator().manual_seed(5)).tolist()
    logits, cache = cp_prefill(model, prompt)
    nxt = model.forward([int(logits.argmax())], cache)[-1]
    if rank == 0:
        ref_cache: dict = {}
        ref = model.forward(prompt, ref_cache)[-1]
        ref_nxt = model.forward([int(ref.argmax())], ref_cache)[-1]
        torch.save({"err": (logits - ref).abs().max().item(), "err2": (nxt - ref_nxt).abs().max().item()}, out_path)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("window", [0, 20])
def test_cp_prefill_model_matches_single_process(window, tmp_path):
    """Whole-model context-parallel prefill (2 gloo ranks) == the single-process forward, and decode
    continues from the gathered cache."""
    path = str(tmp_path / "m.pt")
    mp.spawn(_model_worker, args=(2, _free_port(), window, path), nprocs=2, join=True)
    r = torch.load(path)
    assert r["err"] < 1e-4 and r["err2"] < 1e-4, r
