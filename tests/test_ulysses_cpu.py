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
