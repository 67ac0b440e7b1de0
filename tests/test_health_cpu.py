"""Rank failure detection on the host (no GPU): heartbeats through a TCP store, faults injected
with BARQ_FAULT -- a rank that exits, raises, falls silent, or never joins."""
import socket
import time

import pytest
import torch.multiprocessing as mp
from torch.distributed import TCPStore

from barq_inference_b200.parallel.health import FaultInjector, Heartbeat, RankFailure, parse_faults


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_parse_faults():
    fs = parse_faults("kill:1:5,silence:0:2")
    assert [(f.site, f.rank, f.step) for f in fs] == [("kill", 1, 5), ("silence", 0, 2)]
    with pytest.raises(ValueError):
        parse_faults("explode:0:1")
    inj = FaultInjector(1, "kill:1:5,raise:0:3")
    assert inj.active("kill", 5) and not inj.active("raise", 3)


def _peer(port, spec, q):
    store = TCPStore("127.0.0.1", port, 2, False, timeout=__import__("datetime").timedelta(seconds=30))
    inj = FaultInjector(1, spec)
    hb = Heartbeat(store, 1, 2, period=0.05, timeout=1.0, injector=inj)
    q.put("up")
    for step in range(200):
        inj.on_step(step)  # may exit, raise or silence
        time.sleep(0.05)
    hb.stop()


@pytest.mark.parametrize("spec", ["kill:1:3", "raise:1:3", "silence:1:3"])
def test_dead_peer_is_detected_between_steps(spec):
    port = _port()
    store = TCPStore("127.0.0.1", port, 2, True, wait_for_workers=False)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_peer, args=(port, spec, q))
    p.start()
    assert q.get(timeout=60) == "up"
    hb = Heartbeat(store, 0, 2, period=0.05, timeout=1.0)
    t0 = time.monotonic()
    with pytest.raises(RankFailure):
        for _ in range(400):  # engine steps: check the peers before each one
            hb.check()
            time.sleep(0.05)
    assert time.monotonic() - t0 < 15
    hb.stop()
    p.join(timeout=30)
    if p.is_alive():
        p.kill()


def test_healthy_peer_passes_and_missing_peer_is_reported():
    port = _port()
    store = TCPStore("127.0.0.1", port, 2, True, wait_for_workers=False)
    hb = Heartbeat(store, 0, 2, period=0.05, timeout=0.5)
    with pytest.raises(RankFailure, match="never joined"):
        for _ in range(100):
            hb.check()
            time.sleep(0.05)
    hb.stop()
