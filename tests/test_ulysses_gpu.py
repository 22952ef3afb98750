"""GPU: the Ulysses-sharded hybrid block on 2+ GPUs equals the unsharded block, in the
standard layout (both exchanges) and in every branch-parallel layout, and a model
installed with install_ulysses equals its unsharded forward (on one GPU exactly).

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
    # per clip: two exchanges (peer twice), n - 1 branch-parallel splits, text rows; then
    # the install_ulysses stack, one line per rank
    assert res.stdout.count("rel_l2") == 2 * (4 + n - 1) * n + n


@torch.no_grad()
def test_install_ulysses_single_rank_equals_stack_forward(cuda):
    """install_ulysses on one rank: the installed sharded forward (configure, local rows,
    blocks, gather) gives exactly the stack's own forward."""
    from vdn_b200.block import BlockConfig
    from vdn_b200.stack import HybridStack
    from vdn_b200.ulysses import UlyssesRuntime, install_ulysses
    cfg = BlockConfig(hidden=256, heads=2, head_dim=128, ffn=512, lora_rank=8)
    stack = HybridStack(cfg, depth=2, seed=3, device=cuda)
    g = torch.Generator(device=cuda).manual_seed(5)
    frames, tokens = 4, 64
    x = torch.randn(frames * tokens, 256, device=cuda, generator=g).bfloat16()
    temb = torch.randn(256, device=cuda, generator=g)
    want = stack(x, temb, frames, tokens)
    install_ulysses(stack, UlyssesRuntime(0, 1, 0, cuda, "nccl"))
    got = stack(x, temb, frames, tokens)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
