"""GPU: the tcgen05 block-scaled MXFP8 GEMM against the dequantised oracle.

Mirrors the reference's GEMM oracle (tests/test_paper_stack_mxfp8_ops.py:160-220):
y == bf16(dequant(x) @ dequant(w)^T) + bias within rtol .01 / atol .016, plus the
BASELINE config-1 shapes (M = 32760; N in {15360, 5120, 13824}; K in {5120, 13824})
checked on sampled rows.  Tests run smallest first.
"""
import numpy as np
import pytest
import torch
from torch import nn

from oracle import mxfp8 as omx

pytestmark = pytest.mark.gpu


def unswizzle_index(rows, k, device):
    r = torch.arange(rows, device=device)[:, None]
    c = torch.arange(k // 32, device=device)[None, :]
    return ((r // 128) * (k // 128) + c // 4) * 512 + r % 32 * 16 + (r % 128 // 32) * 4 + c % 4


def dequant(data, scale):
    r, k = data.shape
    natural = scale[unswizzle_index(r, k, data.device)]
    return (data.view(torch.float8_e4m3fn).float().reshape(r, k // 32, 32)
            * torch.exp2(natural.float() - 127)[..., None]).reshape(r, k)


def oracle_gemm(xq, xs, wq, ws, rows, n, bias=None):
    y = (dequant(xq, xs).double() @ dequant(wq, ws).double().T)[:rows, :n]
    y = y.float().bfloat16()
    return y if bias is None else y + bias.bfloat16()


def quantised(m, k, device, seed, scale=1.0, outliers=False):
    from vdn_b200.mxfp8_quant import quantize_activation
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(m, k, device=device, generator=g) * scale
    if outliers:
        idx = torch.randperm(k, device=device, generator=g)[:max(1, k // 100)]
        x[:, idx] *= 50
    return quantize_activation(x.bfloat16())


def run(xq, xs, wq, ws, rows, n, bias=None):
    from vdn_b200.mxfp8_linear import mxfp8_gemm, check_gemm_status
    y = mxfp8_gemm(xq, xs, wq, ws, n, rows=rows, bias=bias)
    torch.cuda.synchronize()
    check_gemm_status(xq.device)
    return y


def test_single_tile(cuda):
    xq, xs = quantised(128, 128, cuda, 1)
    wq, ws = quantised(256, 128, cuda, 2)
    y = run(xq, xs, wq, ws, 128, 256)
    torch.testing.assert_close(y, oracle_gemm(xq, xs, wq, ws, 128, 256), rtol=.01, atol=.016)


@pytest.mark.parametrize("m,n,k", [(128, 256, 512), (256, 384, 256), (384, 512, 1024),
                                   (1024, 1024, 1024), (4096, 2048, 512), (640, 640, 13824 // 27)])
def test_tiles_kblocks_and_persistence(cuda, m, n, k):
    k = (k + 127) // 128 * 128
    xq, xs = quantised(m, k, cuda, m + n)
    wq, ws = quantised(n, k, cuda, k)
    y = run(xq, xs, wq, ws, m, n)
    torch.testing.assert_close(y, oracle_gemm(xq, xs, wq, ws, m, n), rtol=.01, atol=.016)


def test_crop_bias_and_row_stride(cuda):
    from vdn_b200.mxfp8_linear import mxfp8_gemm
    xq, xs = quantised(300, 384, cuda, 5)
    wq, ws = quantised(200, 384, cuda, 6)
    bias = torch.randn(200, device=cuda).bfloat16()
    out = torch.full((290, 256), 7.0, device=cuda, dtype=torch.bfloat16)
    y = mxfp8_gemm(xq, xs, wq, ws, 200, rows=290, bias=bias, out=out[:, :200])
    torch.cuda.synchronize()
    torch.testing.assert_close(y, oracle_gemm(xq, xs, wq, ws, 290, 200, bias), rtol=.01, atol=.016)
    assert bool((out[:, 200:] == 7.0).all())


@pytest.mark.parametrize("shape", [(0, 7, 3), (1, 1, 1), (17, 37, 31), (129, 133, 257), (128, 128, 256)])
@torch.no_grad()
def test_linear_shape_oracle(cuda, shape):
    """Reference test_fused_quant_and_native_gemm_shape_oracle (strided rows, bias)."""
    from vdn_b200.mxfp8_linear import MXFP8Linear
    from vdn_b200.mxfp8_quant import quantize_activation, quantize_cpu
    m, n, k = shape
    torch.manual_seed(42)
    base = torch.randn(m * 2, k, dtype=torch.bfloat16)
    linear = nn.Linear(k, n, bias=True, dtype=torch.bfloat16).eval()
    packed = MXFP8Linear(linear).to(cuda)
    xg = base.to(cuda)[::2]
    q, s = quantize_activation(xg)
    cq, cs = quantize_cpu(base[::2])
    assert torch.equal(q.cpu(), cq) and torch.equal(s.cpu(), cs)
    y = packed(xg)
    assert y.shape == (m, n) and y.dtype == torch.bfloat16 and bool(y.isfinite().all())
    if m:
        oracle = (dequant(q, s) @ dequant(packed.weight_data, packed.weight_scale).T)[:m, :n]
        oracle = oracle.to(torch.bfloat16) + packed.bias
        torch.testing.assert_close(y, oracle, rtol=.01, atol=.016)
    assert torch.equal(packed.weight_data.cpu(), quantize_cpu(linear.weight)[0])


@torch.no_grad()
def test_reject_nonfinite_inputs_and_results(cuda):
    from vdn_b200.mxfp8_linear import MXFP8Linear
    p = MXFP8Linear(nn.Linear(32, 16, bias=False, dtype=torch.bfloat16)).to(cuda)
    x = torch.ones(3, 32, dtype=torch.bfloat16, device=cuda)
    x[0, 0] = float("nan")
    with pytest.raises(ValueError, match="nonfinite MXFP8 activation"):
        p(x)
    x.fill_(1)
    p.weight_data.fill_(127)   # E4M3 NaN: a corrupted compressed weight
    with pytest.raises(ValueError, match="nonfinite MXFP8 result"):
        p(x)


@torch.no_grad()
def test_project_qkv_fused_matches_separate(cuda):
    from vdn_b200.mxfp8_linear import MXFP8Linear, project_qkv
    torch.manual_seed(3)
    projs = [MXFP8Linear(nn.Linear(256, 384, bias=True, dtype=torch.bfloat16), check_finite=False).to(cuda)
             for _ in range(3)]
    x = torch.randn(2, 129, 256, device=cuda, dtype=torch.bfloat16)
    fused = project_qkv(projs, x)
    for got, p in zip(fused, projs):
        assert got.shape == (2, 129, 384)
        assert torch.equal(got, p(x))


@pytest.mark.parametrize("n,k", [(15360, 5120), (5120, 5120), (13824, 5120), (5120, 13824)])
def test_config1_shapes_sampled_rows(cuda, n, k):
    """BASELINE config 1 at full size: M = 32760 activation rows with 1% outlier
    channels x50, weights N(0, 0.02); rows sampled across the M range."""
    m = 32760
    xq, xs = quantised(m, k, cuda, n + k, outliers=True)
    wq, ws = quantised(n, k, cuda, 11, scale=0.02)
    y = run(xq, xs, wq, ws, m, n)
    assert y.shape == (m, n) and bool(torch.isfinite(y).all())
    rows = torch.cat([torch.arange(0, 256), torch.arange(16000, 16128), torch.arange(m - 200, m)]).to(cuda)
    xd = dequant(xq, xs)[rows]
    want = (xd.double() @ dequant(wq, ws).double().T).float().bfloat16()
    torch.testing.assert_close(y[rows], want, rtol=.01, atol=.016)


@pytest.mark.parametrize("rows,row0", [(300, 0), (257, 41), (500, 3)])   # 500: CTA-pair kernel
def test_scatter_epilogue_routes_chunks(cuda, rows, row0):
    """vdn_mxfp8_gemm_scatter: every 128-column chunk lands at its table address,
    row by row, identical to the plain GEMM output (bias included; ragged rows)."""
    from vdn_b200 import _lib
    n, k = 768, 256                       # 6 chunks
    xq, xs = quantised(rows, k, cuda, 31)
    wq, ws = quantised(n, k, cuda, 32, scale=0.05)
    bias = torch.randn(n, device=cuda).bfloat16()
    ref = torch.empty(rows, n, device=cuda, dtype=torch.bfloat16)
    _lib.call("vdn_mxfp8_gemm", _lib.ptr(xq), _lib.ptr(xs), _lib.ptr(wq), _lib.ptr(ws), _lib.ptr(bias),
              xq.shape[0], n, wq.shape[0], k, rows, _lib.ptr(ref), n, None, _lib.stream_of(cuda))
    # destination: [row0 + rows, 3, 2, 128] with chunk c -> slot perm[c]
    total = row0 + rows + 5
    dst = torch.full((total, 6, 128), -7.0, device=cuda).bfloat16()
    perm = [4, 1, 5, 0, 3, 2]
    table = torch.tensor([dst.data_ptr() + perm[c] * 128 * 2 for c in range(6)], dtype=torch.int64,
                         device=cuda)
    _lib.call("vdn_mxfp8_gemm_scatter", _lib.ptr(xq), _lib.ptr(xs), _lib.ptr(wq), _lib.ptr(ws), k,
              _lib.ptr(bias), xq.shape[0], n, wq.shape[0], rows, _lib.ptr(table), 6 * 128, row0, None,
              _lib.stream_of(cuda))
    torch.cuda.synchronize()
    for c in range(6):
        assert torch.equal(dst[row0:row0 + rows, perm[c]], ref[:, c * 128:(c + 1) * 128]), c
    untouched = torch.cat([dst[:row0], dst[row0 + rows:]])
    assert bool((untouched.float() == -7.0).all())


@pytest.mark.parametrize("rows", [300, 500])   # 500 rows pad to 512: the CTA-pair kernel
@pytest.mark.parametrize("act", ["tanh", "none"])
def test_gemm_act_quantize_matches_unfused(cuda, act, rows):
    """vdn_mxfp8_gemm_act_quantize == vdn_mxfp8_gemm (bf16 + bias) followed by the
    GELU quantiser, bit for bit; padded rows come out as zero codes and scales."""
    from vdn_b200 import _lib
    from vdn_b200.mxfp8_kernels import launch_gelu_quantize
    n, k = 384, 512
    xq, xs = quantised(rows, k, cuda, 41)
    wq, ws = quantised(n, k, cuda, 42, scale=0.05)
    bias = torch.randn(n, device=cuda).bfloat16()
    y = torch.empty(rows, n, device=cuda, dtype=torch.bfloat16)
    _lib.call("vdn_mxfp8_gemm", _lib.ptr(xq), _lib.ptr(xs), _lib.ptr(wq), _lib.ptr(ws), _lib.ptr(bias),
              xq.shape[0], n, wq.shape[0], k, rows, _lib.ptr(y), n, None, _lib.stream_of(cuda))
    q = torch.full((xq.shape[0], n), 0x5A, dtype=torch.uint8, device=cuda)
    s = torch.full((xq.shape[0] * n // 32,), 0x5A, dtype=torch.uint8, device=cuda)
    code = _lib.ACT_GELU_TANH if act == "tanh" else 0
    _lib.call("vdn_mxfp8_gemm_act_quantize", _lib.ptr(xq), _lib.ptr(xs), _lib.ptr(wq), _lib.ptr(ws), k,
              _lib.ptr(bias), xq.shape[0], n, wq.shape[0], rows, code, _lib.ptr(q), _lib.ptr(s), None,
              _lib.stream_of(cuda))
    if act == "tanh":
        rq, rs, _ = launch_gelu_quantize(y, approximate="tanh")
    else:
        from vdn_b200.mxfp8_quant import quantize_activation
        rq, rs = quantize_activation(y)
    torch.cuda.synchronize()
    assert torch.equal(q, rq) and torch.equal(s, rs)


@pytest.mark.parametrize("m,n,k", [(4096, 15360, 5120), (32768, 5120, 13824)])
@torch.no_grad()
def test_gemm_matches_torch_blockscaled_mxfp8(cuda, m, n, k):
    """The same codes and swizzled scales through torch's block-scaled MXFP8 GEMM
    (F.scaled_mm, BlockWise1x32 / SWIZZLE_32_4_4: the reference MXFP8Linear's own call,
    src/models/ops/mxfp8_linear.py:89-94): the two fp32-accumulated results agree to a
    few bf16 ulps (different accumulation order only).  Skipped where this torch build
    does not run that GEMM on sm_100."""
    import torch.nn.functional as Fn
    from vdn_b200.mxfp8_linear import mxfp8_gemm
    from vdn_b200.mxfp8_quant import quantize_activation
    g = torch.Generator(device=cuda).manual_seed(m + n)
    x = torch.randn(m, k, device=cuda, generator=g).bfloat16()
    w = (torch.randn(n, k, device=cuda, generator=g) * 0.02).bfloat16()
    xq, xs = quantize_activation(x)
    wq, ws = quantize_activation(w)
    e4, e8 = torch.float8_e4m3fn, torch.float8_e8m0fnu
    try:
        want = Fn.scaled_mm(xq.view(e4), wq.view(e4).T, xs.view(e8), Fn.ScalingType.BlockWise1x32,
                            ws.view(e8), Fn.ScalingType.BlockWise1x32, Fn.SwizzleType.SWIZZLE_32_4_4,
                            Fn.SwizzleType.SWIZZLE_32_4_4, output_dtype=torch.bfloat16)
    except Exception as e:
        pytest.skip(f"torch block-scaled MXFP8 GEMM unavailable on this device: {e!r}"[:200])
    got = mxfp8_gemm(xq, xs, wq, ws, n, rows=m)
    torch.cuda.synchronize()
    want = want[:m, :n].float()
    diff = (got.float() - want).abs()
    # at most one bf16 ulp apart (<= 2^-7 of the value): fp32 sums rounded to bf16
    assert bool((diff <= 2 ** -7 * want.abs() + 1e-4).all()), float(diff.max())
    assert float(diff.norm() / want.norm()) < 1e-3
