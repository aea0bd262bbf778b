"""A bounded device wait that runs out: the peer barrier waits on a flag that nothing sets (an
emulated peer that never arrives), records the timeout in the error word and returns; the host
reads the status and the context stays usable."""
import time

import pytest
import torch

from predicitivecoding_b200 import ops
from predicitivecoding_b200.parallel.health import PeerFailure, check_device_error

pytestmark = pytest.mark.gpu


def test_peer_barrier_timeout_reports_error_and_context_survives():
    own = torch.zeros(64, dtype=torch.int32, device="cuda")
    fake_peer = torch.zeros(64, dtype=torch.int32, device="cuda")      # nobody ever writes our slot here
    table = torch.tensor([own.data_ptr(), fake_peer.data_ptr()], dtype=torch.int64, device="cuda")
    ctr = torch.zeros(1, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    t0 = time.time()
    ops.ext().peer_barrier(table, ctr, 0, 2, err)
    torch.cuda.synchronize()
    dt = time.time() - t0
    assert int(err.item()) == 5 and dt < 15, (int(err.item()), dt)
    assert int(fake_peer[0].item()) == 1          # our arrival was still delivered to the peer's slot
    with pytest.raises(PeerFailure):
        check_device_error(err)
    a = torch.randn(256, 128, device="cuda").to(torch.bfloat16)
    b = torch.randn(128, 128, device="cuda").to(torch.bfloat16)
    c = ops.gemm(a, b, epi=ops.EPI_F32)
    assert torch.allclose(c, a.float() @ b.float().T, atol=0.1, rtol=0.02)
