"""GPU: the Ulysses-sharded hybrid block on 2+ GPUs equals the unsharded block, in the
standard layout (both exchanges) and in every branch-parallel layout.

Runs tests/ulysses_block_check.py under torchrun, one process per GPU, with a
short process-group timeout and an outer `timeout` as the last bound.  Skipped
on a box with fewer than two GPUs.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ulysses_block_matches_unsharded():
    n = 2 if torch.cuda.device_count() < 4 else 4
    here = os.path.dirname(os.path.abspath(__file__))
    cmd = ["timeout", "-k", "30", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}",
           os.path.join(here, "ulysses_block_check.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", PYTHONPATH=os.path.dirname(here))
    res = subprocess.run(cmd, env=env, capture_output=True, text=True)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert res.stdout.count("rel_l2") == 2 * (4 + n - 1) * n
