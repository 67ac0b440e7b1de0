"""NVLS form of the one-shot all-reduce (``allreduce_add_mc_kernel``, multimem.ld_reduce / multimem.st
through NVSwitch) on 2 GPUs against the rank-order sum, and the tiny model's TP=2 logits with it.

Opt-in (``BARQ_TEST_AR_MULTIMEM=1``, needs 2 GPUs bound to an NVLink multicast object): the kernel
is new and its index arithmetic is checked on the CPU (``tests/test_allreduce_mc_cpu.py``) until a
run of this file validates it on NVSwitch GPUs; the product path keeps the peer-load form by default
(``BARQ_AR_MULTIMEM=1`` selects the NVLS one)."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(os.environ.get("BARQ_TEST_AR_MULTIMEM") != "1",
                                 reason="opt-in: BARQ_TEST_AR_MULTIMEM=1 (kernel not yet validated on a GPU)"),
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")]


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      BARQ_AR_MULTIMEM="1")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import torch.distributed as dist

    from barq_inference_b200.parallel.comm import Comm

    try:
        comm = Comm(dev, fused=True, max_elems=1 << 16)
        if not comm._mc_bufs[0]:
            q.put((rank, "skip", "no multicast object on this allocation"))
            return
        g = torch.Generator(device="cpu").manual_seed(rank)
        worst = 0.0
        for it, n in enumerate([4096, 4096 * 3 + 4, 1000, 65536]):
            j = it % 2
            part = torch.randn(n, generator=g).to(dev)
            x = torch.randn(n, generator=torch.Generator().manual_seed(100 + it)).to(dev)
            ref = x + 0
            comm.partial(j, 1, n).view(-1).copy_(part)
            total = part.clone()
            dist.all_reduce(total)
            ref += total
            comm.allreduce_add(j, x)
            comm.check()
            worst = max(worst, (x - ref).abs().max().item())
            xs = [torch.empty_like(x) for _ in range(world)]
            dist.all_gather(xs, x)
            assert all(torch.equal(xs[0], y) for y in xs), "ranks hold different sums"
        q.put((rank, "ok", worst))
    except Exception as e:  # noqa: BLE001
        q.put((rank, "fail", repr(e)))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def test_multimem_allreduce_two_gpus():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(60)
    if any(r[1] == "skip" for r in res):
        pytest.skip(res[0][2])
    assert all(r[1] == "ok" for r in res), res
    assert max(r[2] for r in res) < 1e-4, res
