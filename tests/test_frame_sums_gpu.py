"""GPU: per-frame column sums (vdn_frame_sums), the input of FrameKDAAlpha: the frame
mean of the branch (reference src/models/linear_attention/branch.py:450-452) and the
sequence-parallel frame sums of a row shard (src/inference/utils/ulysses_runtime.py:
606-635).

Against an fp64 sum of the same bf16 rows: the kernel adds in fp32 (eight row groups,
then the groups), so each sum lies within a few fp32 rounding steps of the fp64 one,
bounded here by 2^-20 of the sum of magnitudes.  The order is fixed, so repeated calls
agree bit for bit (the reference replaced an atomic reduction to get that)."""
from types import SimpleNamespace

import pytest
import torch

from vdn_b200 import _lib
from vdn_b200.linear_attention import frame_sums
from vdn_b200.ulysses import UlyssesRuntime

pytestmark = pytest.mark.gpu


def _check(got, x, bounds, divisor):
    got, xd = got.cpu(), x.double()
    for f in range(len(bounds) - 1):
        rows = xd[bounds[f]:bounds[f + 1]]
        want = rows.sum(0) / divisor
        mag = rows.abs().sum(0) / abs(divisor)
        err = (got[f].double() - want).abs()
        assert bool((err <= mag * 2.0 ** -20 + 1e-30).all()), (f, float((err - mag * 2.0 ** -20).max()))


@pytest.mark.parametrize("frames,tokens,width", [(21, 1560, 5120), (3, 7, 8), (5, 100, 264), (1, 1, 512)])
@torch.no_grad()
def test_frame_mean_matches_fp64(cuda, frames, tokens, width):
    g = torch.Generator().manual_seed(frames * 1000 + tokens)
    x = (torch.randn(frames * tokens, width, generator=g) * 3).bfloat16().to(cuda)
    bounds = [f * tokens for f in range(frames + 1)]
    got = frame_sums(x, bounds, tokens)
    _check(got, x.cpu(), bounds, tokens)
    assert torch.equal(got, frame_sums(x, bounds, tokens))


@torch.no_grad()
def test_ragged_ranges_strided_rows_and_empty_frames(cuda):
    g = torch.Generator().manual_seed(5)
    base = torch.randn(300, 1040, generator=g).bfloat16().to(cuda)
    x = base[:, 16:16 + 1000]                       # row stride 1040, 16-byte aligned start
    bounds = [0, 0, 13, 13, 150, 299, 300]          # empty frames 0 and 2
    got = frame_sums(x, bounds, 1.0)
    _check(got, x.cpu(), bounds, 1.0)
    assert not bool(got[0].count_nonzero()) and not bool(got[2].count_nonzero())


@torch.no_grad()
def test_shard_sums_equal_host_path(cuda):
    """UlyssesRuntime.local_frame_sums: the device path (one launch) against the host
    path (one torch sum per frame slice) on the same shard."""
    tpf, frames, prefix = 37, 6, 11
    seq = prefix + frames * tpf
    g = torch.Generator().manual_seed(9)
    x = torch.randn(seq, 64, generator=g).bfloat16()
    for lo, hi in [(0, seq), (0, prefix), (prefix + 5, seq - 20), (seq - 40, seq)]:
        stub = SimpleNamespace(local_start=lo, local_end=hi)
        host = UlyssesRuntime.local_frame_sums(stub, x[lo:hi], frames, tpf, prefix)
        dev = UlyssesRuntime.local_frame_sums(stub, x[lo:hi].to(cuda), frames, tpf, prefix).cpu()
        torch.testing.assert_close(dev, host, rtol=1e-6, atol=1e-5)


def test_argument_checks(cuda):
    lib = _lib.load()
    x = torch.zeros(16, 64, dtype=torch.bfloat16, device=cuda)
    out = torch.empty(2, 64, device=cuda)
    b = (_lib.C.c_int32 * 3)(0, 9, 8)               # decreasing
    rc = lib.vdn_frame_sums(_lib.ptr(x), 64, 16, 64, b, 2, 1.0, _lib.ptr(out), None)
    assert rc == _lib.VDN_ERR_VALUE and b"nondecreasing" in lib.vdn_last_error()
    b = (_lib.C.c_int32 * 3)(0, 8, 16)
    rc = lib.vdn_frame_sums(_lib.ptr(x), 64, 16, 60, b, 2, 1.0, _lib.ptr(out), None)
    assert rc == _lib.VDN_ERR_VALUE                 # width not a multiple of 8
    rc = lib.vdn_frame_sums(_lib.ptr(x), 64, 16, 64, b, 2, 0.0, _lib.ptr(out), None)
    assert rc == _lib.VDN_ERR_VALUE                 # zero divisor
