"""CPU (gloo) gates for the Ulysses runtime: split arithmetic, exact sequence <-> head
routing on ragged shards, the all-gather, and deterministic frame sums.

Mirrors the reference's routing and frame-mean tests
(tests/test_ulysses_allgather.py:22-53, tests/test_ulysses_frame_mean.py:36-66):
three spawned gloo ranks, row counts that leave a short or ragged last shard,
every dtype the block moves, strided sources, inputs left untouched and
contiguous outputs that stay valid across repeated calls.
"""
import multiprocessing
import os
import tempfile
import time
from datetime import timedelta
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist

from vdn_b200.ulysses import UlyssesRuntime, balanced_splits, sequence_splits


def test_sequence_splits_follow_ceil_rule():
    assert sequence_splits(10, 4) == (3, 3, 3, 1)
    assert sequence_splits(9, 3) == (3, 3, 3)
    assert sequence_splits(8, 3) == (3, 3, 2)
    assert sequence_splits(4, 3) == (2, 1, 1)        # ceil leaves nothing last: balanced
    assert sequence_splits(32760, 8) == (4095,) * 8
    assert sequence_splits(7, 1) == (7,)
    for s in range(1, 40):
        for p in range(1, 9):
            if p <= s:
                sp = sequence_splits(s, p)
                assert sum(sp) == s and len(sp) == p and min(sp) > 0
    with pytest.raises(ValueError):
        sequence_splits(0, 2)


def test_balanced_splits():
    assert balanced_splits(10, 4) == (3, 3, 2, 2)
    assert balanced_splits(8, 8) == (1,) * 8
    with pytest.raises(ValueError):
        balanced_splits(3, 4)


def _runtime(rank, world):
    return UlyssesRuntime(rank=rank, world_size=world, local_rank=rank,
                          device=torch.device("cpu"), backend="gloo")


def test_configure_validates():
    rt = _runtime(0, 3)
    with pytest.raises(ValueError):
        rt.configure(9, 4)                          # heads not divisible by ranks
    rt.configure(9, 6)
    assert (rt.local_start, rt.local_end, rt.heads_per_rank) == (0, 3, 2)
    with pytest.raises(RuntimeError):
        rt.configure(12, 6)                          # one geometry per process


def _plain_frame_sums(local_x, local_start, frames, tpf, v0):
    out = torch.zeros(frames, local_x.shape[-1], dtype=torch.float32)
    for f in range(frames):
        a = max(v0 + f * tpf, local_start)
        b = min(v0 + (f + 1) * tpf, local_start + local_x.shape[0])
        if b > a:
            out[f] = local_x[a - local_start:b - local_start].float().sum(0)
    return out


def test_local_frame_sums_exact_and_repeatable():
    tpf, frames, prefix = 6, 5, 4
    seq = prefix + frames * tpf
    torch.manual_seed(0)
    x = torch.randn(seq, 8, dtype=torch.bfloat16)
    for lo, hi in [(0, seq), (0, prefix), (0, prefix + 8), (prefix + 1, seq - 3), (seq - 7, seq)]:
        stub = SimpleNamespace(local_start=lo, local_end=hi)
        first = UlyssesRuntime.local_frame_sums(stub, x[lo:hi], frames, tpf, prefix)
        second = UlyssesRuntime.local_frame_sums(stub, x[lo:hi], frames, tpf, prefix)
        assert torch.equal(first, second)
        torch.testing.assert_close(first, _plain_frame_sums(x[lo:hi], lo, frames, tpf, prefix),
                                   rtol=0, atol=0)


def _worker(rank, world, rendezvous):
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=rendezvous, rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    try:
        heads = 2 * world
        for rows in (4, 8, 9, 10):
            rt = _runtime(rank, world)
            rt.configure(rows, heads)
            lo, hi = rt.local_start, rt.local_end
            hp = rt.heads_per_rank
            prior = []
            for dtype in (torch.float32, torch.bfloat16, torch.float16, torch.int64):
                full = torch.arange(rows * heads * 4).reshape(rows, heads, 4).to(dtype)
                reverse = (-torch.arange(rows * heads * 4).reshape(rows, heads, 4) - 1).to(dtype)
                for strided in (False, True):
                    for method, source, expected in (
                            ("sequence_to_heads", full[lo:hi], full[:, rank * hp:(rank + 1) * hp]),
                            ("heads_to_sequence", reverse[:, rank * hp:(rank + 1) * hp], reverse[lo:hi])):
                        if strided:
                            storage = torch.empty((*source.shape[:-1], source.shape[-1] * 2), dtype=dtype)
                            storage[..., ::2].copy_(source)
                            source = storage[..., ::2]
                        before = source.clone()
                        actual = getattr(rt, method)(source)
                        assert torch.equal(actual, expected), (rank, rows, method, dtype)
                        assert torch.equal(source, before)
                        assert actual.dtype == dtype and actual.is_contiguous()
                        prior.append((actual, expected.clone()))
                    for actual, expected in prior:
                        assert torch.equal(actual, expected)
                # Round trip and the all-gather.
                back = rt.heads_to_sequence(rt.sequence_to_heads(full[lo:hi]))
                assert torch.equal(back, full[lo:hi])
                assert torch.equal(rt.gather_sequence(full[lo:hi].contiguous()), full)
            # Frame sums: the all-reduced per-rank sums are the global per-frame sums.
            tpf = 2
            frames = rows // tpf
            x = torch.linspace(-3, 3, rows * 8).reshape(rows, 8).to(torch.bfloat16)
            sums, work = rt.video_frame_mean_async(x[lo:hi], frames, tpf)
            work.wait()
            want = _plain_frame_sums(x, 0, frames, tpf, 0)
            torch.testing.assert_close(sums, want, rtol=1e-6, atol=1e-5)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_routing_on_gloo_ranks(world):
    with tempfile.TemporaryDirectory() as directory:
        ctx = multiprocessing.get_context("spawn")
        procs = [ctx.Process(target=_worker, args=(r, world, "file://" + directory + "/pg"))
                 for r in range(world)]
        try:
            env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
            old = os.environ.copy()
            os.environ.update(env)
            try:
                for p in procs:
                    p.start()
            finally:
                os.environ.clear()
                os.environ.update(old)
            deadline = time.monotonic() + 120
            for p in procs:
                p.join(max(0, deadline - time.monotonic()))
            assert [p.exitcode for p in procs] == [0] * world
        finally:
            for p in procs:
                if p.is_alive():
                    p.terminate()
                if p.pid is not None:
                    p.join()


# ----------------------------------------------------------- branch-parallel layout
def test_branch_parallel_layout():
    """Rank roles and head ranges of the branch-parallel layout (ulysses_runtime.py:176-251):
    the shipped B200 5 + 3 split of 40 heads, and the argument checks."""
    roles = []
    for rank in range(8):
        rt = _runtime(rank, 8)
        rt.enable_branch_parallel(5)
        rt.configure(32760, 40)
        roles.append((rt.branch_kind, rt.branch_first_head, rt.branch_heads, rt.heads_per_rank))
        assert rt.branch_head_splits == (8, 8, 8, 8, 8, 14, 13, 13)
        assert rt.splits == (4095,) * 8
    assert roles == [("softmax", 8 * r, 8, 8) for r in range(5)] + \
        [("linear", 0, 14, 14), ("linear", 14, 13, 13), ("linear", 27, 13, 13)]
    rt = _runtime(0, 3)
    rt.enable_branch_parallel(2)
    rt.configure(9, 5)                                # heads need not divide the ranks
    assert rt.branch_head_splits == (3, 2, 5)
    for bad in (0, 3, -1, True, 1.0):
        with pytest.raises(ValueError):
            _runtime(0, 3).enable_branch_parallel(bad)
    with pytest.raises(RuntimeError):
        rt.enable_branch_parallel(1)                  # after the first configure
    plain = _runtime(0, 3)
    for attr in ("branch_kind", "branch_head_splits"):
        with pytest.raises(RuntimeError):
            getattr(plain, attr)
    with pytest.raises(RuntimeError):
        plain.branches_to_sequence(torch.zeros(1, 1, 1))
    with pytest.raises(RuntimeError):                 # no dispatch communicators
        rt.dispatch_fields_to_branches_overlapped(*([torch.zeros(3, 5, 4)] * 3), torch.zeros(3, 5),
                                                  *([torch.zeros(3, 5, 4)] * 2), torch.zeros(3, 5),
                                                  torch.zeros(3, 2))


def _branch_worker(rank, world, rendezvous):
    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=rendezvous, rank=rank, world_size=world,
                            timeout=timedelta(seconds=30))
    try:
        d, r = 4, 3
        for softmax_ranks in range(1, world):
            for rows, heads in ((7, world + 2), (10, 2 * world - 1)):
                rt = _runtime(rank, world)
                rt.enable_branch_parallel(softmax_ranks)
                rt.configure(rows, heads)
                lo, hi = rt.local_start, rt.local_end
                g = torch.Generator().manual_seed(rows * 100 + heads)
                for dtype in (torch.bfloat16, torch.float32):
                    fields = [torch.randn(rows, heads, d, generator=g).to(dtype) for _ in range(5)]
                    sq, sk, v, lq, lk = fields
                    sgate, beta = (torch.rand(rows, heads, generator=g).to(dtype) for _ in range(2))
                    shared = torch.randn(rows, r, generator=g).to(dtype)
                    local = [t[lo:hi] for t in (sq, sk, v, sgate, lq, lk, beta, shared)]
                    before = [t.clone() for t in local]
                    packed, got_shared, pending = rt.dispatch_fields_to_branches_overlapped(*local)
                    pending[0].wait()
                    for t, b in zip(local, before):
                        assert torch.equal(t, b)
                    h0, hb = rt.branch_first_head, rt.branch_heads
                    hs = slice(h0, h0 + hb)
                    assert packed.shape == (rows, hb, 3 * d + 1)
                    if rt.branch_kind == "softmax":
                        want = torch.cat([sq[:, hs], sk[:, hs], v[:, hs], sgate[:, hs, None]], -1)
                        assert got_shared is None
                    else:
                        want = torch.cat([lq[:, hs], lk[:, hs], v[:, hs], beta[:, hs, None]], -1)
                        assert torch.equal(got_shared, shared)
                    assert torch.equal(packed, want), (rank, softmax_ranks, rows, heads, dtype)
                    # Reverse exchange: every owner gets all heads of both branches.
                    soft_full = torch.randn(rows, heads, d, generator=g).to(dtype)
                    lin_full = torch.randn(rows, heads, d, generator=g).to(dtype)
                    mine = (soft_full if rt.branch_kind == "softmax" else lin_full)[:, hs]
                    soft_local, lin_local = rt.branches_to_sequence(mine)
                    assert torch.equal(soft_local, soft_full[lo:hi])
                    assert torch.equal(lin_local, lin_full[lo:hi])
                with pytest.raises(ValueError):
                    rt.branches_to_sequence(torch.zeros(rows, rt.branch_heads + 1, d))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [3, 4])
def test_branch_parallel_routing_on_gloo_ranks(world):
    with tempfile.TemporaryDirectory() as directory:
        ctx = multiprocessing.get_context("spawn")
        procs = [ctx.Process(target=_branch_worker, args=(r, world, "file://" + directory + "/pg"))
                 for r in range(world)]
        old = os.environ.copy()
        os.environ["CUDA_VISIBLE_DEVICES"] = ""
        try:
            for p in procs:
                p.start()
        finally:
            os.environ.clear()
            os.environ.update(old)
        try:
            deadline = time.monotonic() + 180
            for p in procs:
                p.join(max(0, deadline - time.monotonic()))
            assert [p.exitcode for p in procs] == [0] * world
        finally:
            for p in procs:
                if p.is_alive():
                    p.terminate()
                if p.pid is not None:
                    p.join()


# ------------------------------------------------------------------- install_ulysses
def _small_stack(heads=2, depth=2):
    from vdn_b200.block import BlockConfig
    from vdn_b200.stack import HybridStack
    cfg = BlockConfig(hidden=128 * heads, heads=heads, head_dim=128, ffn=256, lora_rank=4)
    return HybridStack(cfg, depth=depth, seed=1, device="cpu")


def test_install_ulysses_refusals():
    """The reference's checks (src/inference/utils/ulysses.py:717-764)."""
    from vdn_b200.ulysses import install_ulysses
    with pytest.raises(ValueError, match="requires a HybridAttention checkpoint"):
        install_ulysses(torch.nn.Linear(2, 2), _runtime(0, 2))
    with pytest.raises(ValueError, match="attention heads are not divisible by 3 ranks"):
        install_ulysses(_small_stack(heads=2), _runtime(0, 3))
    mixed = _small_stack(heads=2)
    mixed.blocks[1].cfg = type(mixed.cfg)(hidden=512, heads=4, head_dim=128, ffn=256)
    with pytest.raises(ValueError, match="same attention head count"):
        install_ulysses(mixed, _runtime(0, 2))
    with pytest.raises(ValueError, match="softmax_ranks must lie in"):
        install_ulysses(_small_stack(heads=2), _runtime(0, 2), softmax_ranks=2)


def test_install_ulysses_binds_runtime_and_forwards():
    from vdn_b200.ulysses import install_ulysses
    stack = _small_stack(heads=2)
    rt = _runtime(1, 2)
    install_ulysses(stack, rt)
    assert stack._ulysses_runtime is rt
    assert all(b._ulysses_runtime is rt for b in stack.transformer_blocks)
    assert stack.forward.__func__.__name__ == "_ulysses_transformer_forward"
    assert stack.blocks[0].forward.__func__.__name__ == "_ulysses_block_forward"
    x = torch.zeros(4 * 8, 256, dtype=torch.bfloat16)
    with torch.enable_grad(), pytest.raises(RuntimeError, match="inference-only"):
        stack(x, torch.zeros(256), 4, 8)
    with torch.no_grad(), pytest.raises(ValueError, match="text_rows \\+ frames \\* tokens"):
        stack(x, torch.zeros(256), 5, 8)
    brt = _runtime(0, 2)
    install_ulysses(_small_stack(heads=2), brt, softmax_ranks=1)
    assert brt.branch_parallel and brt.softmax_ranks == 1
