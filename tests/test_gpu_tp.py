"""Tensor parallel (attention TP x MoE EP) on 2 GPUs vs the same model on one GPU.

Runs 2 NCCL ranks as child processes (skipped with fewer than 2 GPUs).  Three communication modes:
"push" (decode: the all-reduce fused into the row-parallel streaming GEMV; otherwise the one-shot
kernel), "oneshot" (symmetric memory, csrc/kernels/allreduce.cu), "sp" (prefill: sequence-parallel
residual with the reduce-scatter fused into the row-parallel tcgen05 GEMM and the all-gather into
the next column-parallel GEMM, csrc/kernels/tp_fused.cu; decode: as "push") and the NCCL baseline.
"tiny-sp" is the tiny config widened to 8 heads / 8 KV heads (shardable up to TP=8) with an FFN width
that keeps gate|up interleaved after sharding, which the sequence-parallel path needs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
needs2 = pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")


def _step(runner, toks, start, table, decode):
    from barq_inference_b200.models.runner import StepInput

    T = len(toks)
    pos = list(range(start, start + T))
    slots = [table[p // 16] * 16 + p % 16 for p in pos]
    dev = runner.device
    d = lambda a, dt: torch.tensor(a, dtype=dt, device=dev)  # noqa: E731
    inp = StepInput(d(toks, torch.int32), d(pos, torch.int32), d(slots, torch.int64), d([table], torch.int32),
                    d([start + T], torch.int32), d([T - 1], torch.int64), decode,
                    q_start=d([0, T], torch.int32), max_q=T)
    return runner.forward(inp)[0].float().cpu()


def _logits(runner, prompt, steps=3):
    table = list(range(1, 10))
    out = [_step(runner, prompt, 0, table, False)]
    pos = len(prompt)
    for _ in range(steps):
        t = int(out[-1].argmax())
        out.append(_step(runner, [t], pos, table, True))
        pos += 1
    return torch.stack(out)


def _worker(rank, world, port, name, mode, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    from barq_inference_b200.models import POLICIES, preset, random_tensors
    from barq_inference_b200.models.runner import LlamaRunner
    from barq_inference_b200.parallel.comm import Comm
    from barq_inference_b200.parallel.tp import shard_config, shard_tensors

    import dataclasses

    wide = dict(hidden=512, n_heads=8, n_kv_heads=8, head_dim=64, ffn=1024)
    cfg = (dataclasses.replace(preset("tiny"), **wide) if name == "tiny-sp" else
           dataclasses.replace(preset("tiny-moe"), n_experts=8, **wide) if name == "tiny-moe-sp" else preset(name))
    full = random_tensors(cfg, POLICIES["tiny-ds" if cfg.is_mla else "tiny"], seed=4)
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, cfg.vocab, (20,), generator=g).tolist()
    comm = Comm(dev, fused=mode != "nccl", max_elems=64 * cfg.hidden,
                hidden=cfg.hidden if mode in ("push", "sp") else 0, sp_tokens=64 if mode == "sp" else 0,
                ep_experts=cfg.n_experts if mode == "sp" else 0, ep_topk=cfg.n_experts_used)
    if mode == "sp":
        comm.sp_min_tokens = 9  # the 20-token prompt runs sequence-parallel
    shard, info = shard_tensors(cfg, full, rank, world)
    if cfg.is_mla:  # DeepSeek-V2: heads split, latent path replicated
        from barq_inference_b200.models.deepseek2 import DeepseekV2Runner

        r = DeepseekV2Runner(cfg, shard, dev, tp=info, comm=comm)
    else:
        r = LlamaRunner(shard_config(cfg, world), shard, dev, tp=info, comm=comm)
    r.allocate_kv(32)
    tp_logits = _logits(r, prompt)
    comm.check()
    pushes = int(comm.push_epoch.sum()) if mode in ("push", "sp") else -1
    if mode in ("push", "sp"):  # the fused GEMV all-reduce ran on the decode steps (epochs advance per call)
        assert pushes > 0, pushes
    if mode == "sp":  # the 20-token prefill ran sequence-parallel: both sites advanced once per layer
        assert int(comm.sp_epoch[0]) == cfg.n_layers and int(comm.sp_epoch[1]) == cfg.n_layers + 1, comm.sp_epoch
        if cfg.n_experts:  # ... and every MoE layer went through the expert all-to-all
            assert int(comm.ep_epoch[0]) == cfg.n_layers, comm.ep_epoch
    if rank == 0:
        if cfg.is_mla:
            from barq_inference_b200.models.deepseek2 import DeepseekV2Runner

            ref = DeepseekV2Runner(cfg, full, dev)
        else:
            ref = LlamaRunner(cfg, full, dev)
        ref.allocate_kv(32)
        q.put(("ok", (tp_logits - _logits(ref, prompt)).abs().max().item()))
    comm.barrier()
    import torch.distributed as dist

    dist.destroy_process_group()


def _run_tp(world, name, mode):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_worker, args=(r, world, port, name, mode, q)) for r in range(world)]
    for p in ps:
        p.start()
    status, err = q.get(timeout=300)
    for p in ps:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in ps)
    assert err < 2e-2, err


@needs2
@pytest.mark.parametrize("name", ["tiny", "tiny-moe"])
@pytest.mark.parametrize("mode", ["push", "oneshot", "nccl"])
def test_tp2_matches_single_gpu(name, mode):
    _run_tp(2, name, mode)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_sequence_parallel_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _run_tp(world, "tiny-sp", "sp")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_expert_parallel_all_to_all_matches_single_gpu(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    _run_tp(world, "tiny-moe-sp", "sp")


@needs2
@pytest.mark.parametrize("mode", ["oneshot", "nccl"])
def test_tp2_deepseek_mla_matches_single_gpu(mode):
    """DeepSeek-V2 (MLA + shared / routed experts) with its 16 heads split over 2 ranks."""
    _run_tp(2, "tiny-ds", mode)


def _pp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import datetime

    import torch.distributed as dist

    from barq_inference_b200.models import POLICIES, preset, random_tensors
    from barq_inference_b200.models.runner import LlamaRunner
    from barq_inference_b200.parallel.pp import PPInfo, shard_pp, stage_layers

    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    cfg = preset("tiny")
    full = random_tensors(cfg, POLICIES["tiny"], seed=4)
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, cfg.vocab, (20,), generator=g).tolist()
    l0, l1 = stage_layers(cfg.n_layers, world)[rank]
    r = LlamaRunner(cfg, shard_pp(full, cfg.n_layers, rank, world), dev, pp=PPInfo(rank, world, l0, l1))
    r.allocate_kv(32)
    pp_logits = _logits(r, prompt)
    if rank == 0:
        if cfg.is_mla:
            from barq_inference_b200.models.deepseek2 import DeepseekV2Runner

            ref = DeepseekV2Runner(cfg, full, dev)
        else:
            ref = LlamaRunner(cfg, full, dev)
        ref.allocate_kv(32)
        q.put(("ok", (pp_logits - _logits(ref, prompt)).abs().max().item()))
    dist.barrier()
    dist.destroy_process_group()


@needs2
def test_pp2_matches_single_gpu():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_pp_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    status, err = q.get(timeout=300)
    for p in ps:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in ps)
    assert err < 1e-3, err
