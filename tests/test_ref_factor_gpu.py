"""GPU: the factor stage against the reference's own sm_100 factor kernel
(src/models/ops/csrc/vdn_delta_factors.cuh:200-306, the FFMA2 Gauss-Jordan kernel its
paper_delta_factors launches), compiled from the reference checkout into oracle/_ref/
by oracle/build_ref.py and run on the same inputs.

* parity: paper_delta_factors (this library's T / J kernel) and the reference kernel
  each against fp64 at the factor bars (rel-L2 1e-5 for T, 3e-5 for J), and the two
  against each other;
* timing, reported and not asserted: both T / J kernels on the config-2/3 factor batch
  (21 frames x 40 heads = 840 matrices, statistics of 1560-token frames), and the
  forward path's own factor stage, which writes only the split inverse and leaves
  B (I + A)^-1 to the tensor-core scan (timed with it).  CUDA events on the launching
  stream, L2 flushed (256 MB write) before every launch, median of 20 after 3 warm-up
  launches.  `pytest -s` prints one REF_FACTOR_TIMING line.
"""
import ctypes
import json
import statistics
from pathlib import Path

import pytest
import torch
import torch.nn.functional as F

from helpers import rel_l2

pytestmark = pytest.mark.gpu

LIB = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libref_factors.so"


@pytest.fixture(scope="module")
def ref_lib():
    if not LIB.exists():
        pytest.skip("reference factor kernel not built (python -m oracle.build_ref)")
    lib = ctypes.CDLL(str(LIB))
    lib.ref_delta_factors.restype = ctypes.c_int
    lib.ref_delta_factors.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64, ctypes.c_void_p]
    return lib


def _ref_factors(lib, A, B, alpha, T=None, J=None):
    T = torch.empty_like(A) if T is None else T
    J = torch.empty_like(B) if J is None else J
    n = A.numel() // (128 * 128)
    rc = lib.ref_delta_factors(A.data_ptr(), B.data_ptr(), alpha.data_ptr(), T.data_ptr(), J.data_ptr(), n,
                               torch.cuda.current_stream(A.device).cuda_stream)
    assert rc == 0, rc
    return T, J


def _statistics(frames, heads, tokens, device, seed=0):
    """A = (k beta)^T k, B = (v beta)^T k of SiLU + L2 features, alpha in (0.1, 1): the
    factor inputs of one VDA call, built on the device in fp32."""
    g = torch.Generator(device=device).manual_seed(seed)
    shape = (frames, heads, tokens, 128)
    k = F.normalize(F.silu(torch.randn(shape, generator=g, device=device)), dim=-1)
    v = F.silu(torch.randn(shape, generator=g, device=device))
    beta = torch.sigmoid(torch.randn(shape[:-1], generator=g, device=device))
    alpha = torch.rand(frames, heads, 128, generator=g, device=device) * 0.9 + 0.1
    kb = k * beta.unsqueeze(-1)
    A = kb.transpose(-1, -2) @ k
    A = 0.5 * (A + A.transpose(-1, -2))
    B = (v * beta.unsqueeze(-1)).transpose(-1, -2) @ k
    return A.contiguous(), B.contiguous(), alpha.contiguous()


def _fp64(A, B, alpha):
    a, b = A.double().cpu(), B.double().cpu()
    system = torch.eye(128, dtype=torch.float64) + a
    inv = torch.linalg.inv(system)
    return alpha.double().cpu()[..., :, None] * inv, b @ inv


@torch.no_grad()
@pytest.mark.parametrize("frames,heads,tokens", [(1, 1, 16), (3, 5, 1560)])
def test_factors_match_reference_kernel(cuda, ref_lib, frames, heads, tokens):
    from vdn_b200.paper_factor import paper_delta_factors
    torch.backends.cuda.matmul.allow_tf32 = False
    A, B, alpha = _statistics(frames, heads, tokens, cuda)
    rt, rj = _ref_factors(ref_lib, A, B, alpha)
    t, j = paper_delta_factors(A, B, alpha)
    torch.cuda.synchronize()
    et, ej = _fp64(A, B, alpha)
    for got, want, lim in ((rt, et, 1e-5), (rj, ej, 3e-5), (t, et, 1e-5), (j, ej, 3e-5)):
        assert bool(torch.isfinite(got).all())
        assert rel_l2(got.double().cpu().numpy(), want.numpy()) < lim
    assert rel_l2(t.double().cpu().numpy(), rt.double().cpu().numpy()) < 1e-5
    assert rel_l2(j.double().cpu().numpy(), rj.double().cpu().numpy()) < 3e-5


def _median_ms(fn, device, reps=20, warm=3):
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    for _ in range(warm):
        fn()
    times = []
    for _ in range(reps):
        flush.fill_(reps & 0xFF)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    return statistics.median(times)


@torch.no_grad()
def test_factor_timing_config3_batch(cuda, ref_lib):
    from vdn_b200 import _lib
    from vdn_b200.linear_attention import SPLIT_INVERSE_BYTES, split_inverse_values
    torch.backends.cuda.matmul.allow_tf32 = False
    frames, heads = 21, 40
    A, B, alpha = _statistics(frames, heads, 1560, cuda, seed=1)
    n = frames * heads
    stream = _lib.stream_of(cuda)
    T, J = torch.empty_like(A), torch.empty_like(B)
    T2, J2 = torch.empty_like(A), torch.empty_like(B)
    planes = torch.empty(frames, heads, SPLIT_INVERSE_BYTES, dtype=torch.uint8, device=cuda)
    prefix, suffix = torch.empty_like(B), torch.empty_like(B)
    status = torch.zeros(1, dtype=torch.int32, device=cuda)

    def ref():
        _ref_factors(ref_lib, A, B, alpha, T, J)

    def ours_tj():
        _lib.call("vdn_delta_factors", _lib.ptr(A), _lib.ptr(B), _lib.ptr(alpha), n, 128, _lib.ptr(T2),
                  _lib.ptr(J2), stream)

    def ours_inverse():
        _lib.call("vdn_vda_factor_inverse", _lib.ptr(A), n, _lib.ptr(planes), stream)

    def ours_scan():
        _lib.call("vdn_vda_scan_tc", _lib.ptr(planes), _lib.ptr(B), _lib.ptr(alpha), None, frames, heads,
                  _lib.ptr(prefix), _lib.ptr(suffix), _lib.ptr(status), stream)

    res = {"matrices": n, "ref_factor_ms": _median_ms(ref, cuda), "tj_factor_ms": _median_ms(ours_tj, cuda),
           "inverse_ms": _median_ms(ours_inverse, cuda), "scan_ms": _median_ms(ours_scan, cuda)}
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # The timed launches computed the same factors.
    assert rel_l2(T2.double().cpu().numpy(), T.double().cpu().numpy()) < 1e-5
    inv = split_inverse_values(planes)
    assert rel_l2((alpha[..., :, None] * inv).double().cpu().numpy(), T.double().cpu().numpy()) < 1e-5
    res["ref_over_tj"] = res["ref_factor_ms"] / res["tj_factor_ms"]
    res["ref_over_inverse"] = res["ref_factor_ms"] / res["inverse_ms"]
    print("REF_FACTOR_TIMING " + json.dumps({k: round(v, 4) if isinstance(v, float) else v
                                               for k, v in res.items()}))
