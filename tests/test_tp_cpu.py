"""Tensor/expert-parallel host logic on the CPU: GGUF-level sharding identities and the NCCL-path
row-parallel reduction (rank 0 adds, others store, all-reduce) over gloo with 2 processes."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from barq_inference_b200.models import POLICIES, preset, random_tensors
from barq_inference_b200.models.reference import dequant_tensor
from barq_inference_b200.parallel.tp import shard_config, shard_tensors


# K-quant rows split on 256-column blocks: the test-sized models use 32-column Q4_0 blocks so that
# their narrow (256-wide) row-parallel weights can be split at all
@pytest.mark.parametrize("name,world", [("tiny", 2), ("tiny-moe", 2)])
def test_shards_reassemble_to_full_tensors(name, world):
    cfg = preset(name)
    full = random_tensors(cfg, POLICIES["tiny"], seed=1)
    shards = [shard_tensors(cfg, full, r, world) for r in range(world)]
    for n, pt in full.items():
        parts = [dequant_tensor(s[0][n]) for s in shards]
        ref = dequant_tensor(pt)
        short = n.split(".", 2)[-1]
        if short in ("attn_output.weight", "ffn_down.weight"):
            got = torch.cat(parts, -1)
        elif parts[0].numel() == ref.numel():  # replicated (norms, router, embeddings)
            assert all(torch.equal(p, ref) for p in parts), n
            continue
        elif n == "token_embd.weight" and "output.weight" in full:
            got = parts[0]
        else:
            got = torch.cat(parts, 0)
        assert torch.equal(got.reshape(ref.shape), ref), n
    infos = [s[1] for s in shards]
    if cfg.is_moe:
        assert [i.expert0 for i in infos] == [r * cfg.n_experts // world for r in range(world)]
    assert sum(i.vocab_local for i in infos) == cfg.vocab
    sc = shard_config(cfg, world)
    assert sc.n_heads * world == cfg.n_heads and sc.ffn * world == cfg.ffn


def test_shard_rejects_unaligned_columns():
    cfg = preset("tiny")
    full = random_tensors(cfg, POLICIES["tiny"], seed=1)
    with pytest.raises(ValueError):
        shard_tensors(cfg, full, 0, 3)  # 4 heads are not divisible by 3


class _GlooComm:
    fused = False

    def __init__(self, rank, world):
        self.rank, self.world = rank, world

    def all_reduce(self, x):
        dist.all_reduce(x)
        return x


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from barq_inference_b200.models.runner import LlamaRunner

    r = LlamaRunner.__new__(LlamaRunner)
    r.comm = _GlooComm(rank, world)
    x = torch.arange(8, dtype=torch.float32)  # replicated residual
    partial = torch.full((8,), float(rank + 1))

    def fn(mode, out):
        from barq_inference_b200.ops import EPI_ADD_F32

        if mode == EPI_ADD_F32:
            out += partial
        else:
            out.copy_(partial)
    r._row_parallel(0, fn, x)
    q.put((rank, x.tolist()))
    dist.destroy_process_group()


def test_row_parallel_reduction_gloo():
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
    want = [float(i) + 1 + 2 for i in range(8)]  # residual + sum of partials (1 + 2)
    assert res[0] == want and res[1] == want


def test_pipeline_stage_split_and_tensor_filter():
    from barq_inference_b200.parallel.pp import shard_pp, stage_layers

    assert stage_layers(32, 4) == [(0, 8), (8, 16), (16, 24), (24, 32)]
    assert stage_layers(5, 2) == [(0, 3), (3, 5)]
    with pytest.raises(ValueError):
        stage_layers(2, 3)
    cfg = preset("tiny")
    full = random_tensors(cfg, POLICIES["tiny"], seed=1)
    s0, s1 = (shard_pp(full, cfg.n_layers, s, 2) for s in range(2))
    assert "token_embd.weight" in s0 and "output_norm.weight" not in s0
    assert "output_norm.weight" in s1 and "blk.0.attn_q.weight" not in s1
    assert {k for k in s0 if k.startswith("blk.")} | {k for k in s1 if k.startswith("blk.")} == \
        {k for k in full if k.startswith("blk.")}


def _grid_worker(rank, world, port, out_path):
    from barq_inference_b200.parallel.pp import PPInfo, grid_groups

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    stage, t, tpg, ppg = grid_groups(2, 2)
    x = torch.tensor([float(rank)])
    dist.all_reduce(x, group=tpg)  # sum over the two tensor ranks of this stage
    info = PPInfo(stage, 2, 0, 1, tp=2, tp_rank=t, group=ppg)
    logits = torch.tensor([100.0 + rank]) if info.is_last else torch.zeros(1)
    info.broadcast_logits(logits)  # from the last stage's rank with the same tensor rank
    h = torch.tensor([10.0 * rank])
    if stage == 0:
        info.send(h)
    else:
        info.recv(h)
    torch.save({"stage": stage, "t": t, "tp_sum": x.item(), "logits": logits.item(), "h": h.item(),
                "dst": info.global_rank(1)}, f"{out_path}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


def test_tp_pp_grid_groups(tmp_path):
    """tp=2 x pp=2 over 4 gloo ranks: rank = stage * tp + t; tensor-parallel sums stay inside a stage,
    hidden states go to the same tensor rank of the next stage, logits come from the last stage."""
    import socket as _s

    with _s.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "g")
    mp.spawn(_grid_worker, args=(4, port, path), nprocs=4, join=True)
    r = [torch.load(f"{path}.{i}") for i in range(4)]
    assert [(x["stage"], x["t"]) for x in r] == [(0, 0), (0, 1), (1, 0), (1, 1)]
    assert [x["tp_sum"] for x in r] == [1.0, 1.0, 5.0, 5.0]
    assert [x["logits"] for x in r] == [102.0, 103.0, 102.0, 103.0]
    assert [x["h"] for x in r] == [0.0, 10.0, 0.0, 10.0]  # stage 1 received its stage-0 peer's states


def test_mla_shards_heads_and_keeps_latent_path_whole():
    """DeepSeek-V2 tensor parallel: query / kv_b rows and output columns by head, the latent
    projections, dense FFN and shared experts whole, routed experts by expert; the shards' query
    rows and output columns reassemble the full tensors."""
    import torch

    from barq_inference_b200.models import POLICIES, preset, random_tensors
    from barq_inference_b200.parallel.tp import shard_tensors

    cfg = preset("tiny-ds")
    full = random_tensors(cfg, POLICIES["tiny-ds"], seed=4)
    shards = [shard_tensors(cfg, full, r, 2) for r in range(2)]
    for r, (sh, info) in enumerate(shards):
        assert (info.head0, info.n_heads_local) == (8 * r, 8)
        assert sh["blk.1.attn_kv_a_mqa.weight"] is full["blk.1.attn_kv_a_mqa.weight"]
        assert sh["blk.0.ffn_down.weight"] is full["blk.0.ffn_down.weight"]
        assert sh["blk.1.ffn_down_shexp.weight"] is full["blk.1.ffn_down_shexp.weight"]
        assert sh["blk.1.ffn_gate_exps.weight"].shape[0] == 2 and info.expert0 == 2 * r
    q = torch.cat([shards[r][0]["blk.1.attn_q.weight"].data for r in range(2)])
    assert torch.equal(q, full["blk.1.attn_q.weight"].data)
    o = torch.cat([shards[r][0]["blk.1.attn_output.weight"].data for r in range(2)], 1)
    assert torch.equal(o, full["blk.1.attn_output.weight"].data)
