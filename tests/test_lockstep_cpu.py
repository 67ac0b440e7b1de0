"""Multi-rank serving in lockstep over gloo: rank 0's engine publishes each step's new requests
through the store, rank 1 replays them; both ranks take the same steps and produce the same tokens
(engines with the CPU paged runner; sampled requests included)."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank, world, port, out_path):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import test_engine_paged_cpu as H
    import barq_inference_b200.engine.engine as engine_mod
    from barq_inference_b200.engine.sampling_params import SamplingParams
    from barq_inference_b200.models import POLICIES, preset, random_tensors
    from barq_inference_b200.parallel.lockstep import LockstepLeader, follower_loop
    from torch.distributed.distributed_c10d import _get_default_store

    def sample(logits, temp, topk, topp, minp, seeds, steps, **kw):  # seeded, so ranks must agree on seeds
        g = torch.Generator().manual_seed(int(seeds[0]) * 7919 + int(steps[0]))
        probs = torch.softmax(logits.float() / 0.8, -1)
        return torch.multinomial(probs, 1, generator=g)[:, 0].to(torch.int32), None

    engine_mod.ops.sample = sample
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    store = _get_default_store()
    cfg = preset("tiny", n_layers=1, vocab=400, max_ctx=256)
    t = random_tensors(cfg, POLICIES["tiny"], seed=1)
    eng = H._engine(cfg, t, num_blocks=64, max_num_batched_tokens=32, max_num_seqs=3)
    if rank == 0:
        lead = LockstepLeader(eng, store)
        seqs = [lead.add_request([1, 2, 3, 4, 5][: 2 + i], SamplingParams(max_tokens=6 + i, temperature=0.8))
                for i in range(3)]
        for _ in range(2):
            lead.step()
        seqs.append(lead.add_request(list(range(10, 40)), SamplingParams(max_tokens=5, temperature=0.8)))
        while lead.has_work():
            lead.step()
        lead.stop()
        toks = [s.output for s in seqs]
        n = lead.k - 1
    else:
        seqs = []
        n = follower_loop(eng, store, collect=seqs)
        toks = [s.output for s in seqs]
    torch.save({"steps": n, "toks": toks, "step_count": eng.step_count}, f"{out_path}.{rank}")
    dist.barrier()
    dist.destroy_process_group()


def test_leader_and_follower_take_the_same_steps(tmp_path):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    path = str(tmp_path / "r")
    mp.spawn(_worker, args=(2, port, path), nprocs=2, join=True)
    a, b = torch.load(f"{path}.0"), torch.load(f"{path}.1")
    assert a["step_count"] == b["step_count"] == a["steps"] == b["steps"] > 0
    assert [len(x) for x in a["toks"]] == [6, 7, 8, 5]
    assert a["toks"] == b["toks"]  # sampled with per-sequence seeds: the follower drew the same tokens
