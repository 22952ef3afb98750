"""GPU failure detection without a GPU fault: bounded waits return an error status.

The Ulysses peer fence waits (acquire loads, 2 s limit) for every rank's flag.
Here a two-rank fence runs on ONE GPU with a "peer" flag array that nothing
ever writes: the wait runs out, the kernel returns, the status word reads
VDN_ERR_TIMEOUT, and the context stays usable (a later launch succeeds).
No trap, no fault, no second kernel waiting on this one.
"""
import ctypes as C

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_fence_times_out_with_status(cuda):
    from vdn_b200 import _lib
    mine = torch.zeros(16, dtype=torch.int64, device=cuda)     # this rank's flags + counter
    peer = torch.zeros(16, dtype=torch.int64, device=cuda)     # a "peer" that never arrives
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    flags = (C.c_void_p * 2)(mine.data_ptr(), peer.data_ptr())
    counter = C.c_void_p(mine.data_ptr() + 8 * 8)
    _lib.call("vdn_peer_fence", 2, flags, C.c_void_p(mine.data_ptr()), 0, counter, _lib.ptr(status),
              _lib.stream_of(cuda))
    torch.cuda.synchronize()
    assert int(status.item()) == _lib.VDN_ERR_TIMEOUT
    # Rank 0 published epoch 1 into its own slot and into the "peer" array.
    assert int(mine[0].item()) == 1 and int(peer[0].item()) == 1
    assert int(mine[8].item()) == 1                              # the counter advanced
    # The context is intact.
    x = torch.randn(1024, device=cuda)
    assert torch.isfinite(x.sum()).item()


def test_fence_single_rank_completes(cuda):
    from vdn_b200 import _lib
    mine = torch.zeros(16, dtype=torch.int64, device=cuda)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)
    flags = (C.c_void_p * 1)(mine.data_ptr())
    for epoch in (1, 2, 3):
        _lib.call("vdn_peer_fence", 1, flags, C.c_void_p(mine.data_ptr()), 0,
                  C.c_void_p(mine.data_ptr() + 64), _lib.ptr(status), _lib.stream_of(cuda))
        torch.cuda.synchronize()
        assert int(status.item()) == 0 and int(mine[8].item()) == epoch
