"""Failure detection of the fused all-reduce without a GPU fault: a one-process 'world of 2' whose
second rank never signals.  The kernel's bounded barrier wait must run out (0.5 s), record the
error word, leave x unchanged and return; the host check must raise."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_fused_allreduce_peer_timeout_is_reported():
    from barq_inference_b200.ops import require_ext

    C = require_ext()
    C.gemm_clear_error()
    n = 4096
    x = torch.arange(n, dtype=torch.float32, device="cuda")
    mine = torch.ones(n, device="cuda")
    fake_peer = torch.ones(n, device="cuda")          # "rank 1's" partial: never read
    flags0 = torch.zeros(64 * 8, dtype=torch.int32, device="cuda")  # my flag area: rank 1 never writes
    flags1 = torch.zeros(64 * 8, dtype=torch.int32, device="cuda")  # "rank 1's" flag area (receives my signal)
    epoch = torch.zeros(64, dtype=torch.int32, device="cuda")
    before = x.clone()
    C.allreduce_add(x, [mine.data_ptr(), fake_peer.data_ptr()], [flags0.data_ptr(), flags1.data_ptr()], epoch, 0,
                    4, 0.5, 0, 0)
    torch.cuda.synchronize()
    err = C.gemm_error()
    assert err & 0xF00 == 0x300 and err & 0xFF == 1, hex(err)
    assert torch.equal(x, before)                      # no partial sum applied
    assert int(flags1[:4 * 8].view(4, 8)[:, 0].min()) == 1  # our signal reached the (fake) peer
    assert int(epoch[:4].min()) == 1                   # epochs advanced: ranks stay aligned
    from barq_inference_b200.parallel.comm import Comm

    c = Comm.__new__(Comm)
    with pytest.raises(RuntimeError):
        c.check()
    C.gemm_clear_error()
    # the context is still usable
    y = torch.ones(8, device="cuda") * 2
    assert float(y.sum()) == 16.0
