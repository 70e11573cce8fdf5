"""A device-side bounded wait that runs out records an error the host reads, and the context
stays usable.  The peer barrier kernel waits for a flag that nothing sets (both "ranks" are
buffers of this GPU, so no peer memory is touched); after its 10 ms limit it records code 3 at
the waiting slot and returns."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_barrier_times_out_and_reports():
    from nexttransformer_b200.ops._ext import ext
    lib = ext()
    torch.cuda.synchronize()
    lib.clear_comm_errors()
    assert lib.read_comm_errors()[0] == 0
    pads = [torch.zeros(256, dtype=torch.int32, device="cuda") for _ in range(2)]
    table = torch.tensor([p.data_ptr() for p in pads], dtype=torch.int64, device="cuda")
    t0 = time.monotonic()
    lib.p2p_barrier(table, 0, 2, 1, 0.01)      # rank 1 never arrives
    torch.cuda.synchronize()
    elapsed = time.monotonic() - t0
    code, where = lib.read_comm_errors()
    assert code == 3 and where == 0xA01, (code, hex(where))
    assert elapsed < 5.0
    assert int(pads[1][0]) == 1          # rank 0 did announce itself in the other pad
    x = torch.randn(4096, device="cuda")  # the context is still usable
    assert torch.isfinite((2 * x).sum())
    lib.clear_comm_errors()
    assert lib.read_comm_errors()[0] == 0
