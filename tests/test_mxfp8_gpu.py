"""GPU: the sm_100a MXFP8 quantiser and producers against the reference fixtures and
the oracle (bit-exact codes and scales), mirroring the reference's GPU oracles
tests/test_paper_stack_mxfp8_ops.py:160-220 and tests/test_tp_producers.py:104-131."""
import numpy as np
import pytest
import torch

from oracle import mxfp8 as mx
from helpers import bf16_tensor, bits_of

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["cfg0", "outlier"] + [f"shape{i}" for i in range(6)])
def test_device_quantiser_bit_exact_vs_reference(cuda, mxfp8_golden, case):
    from vdn_b200.mxfp8_quant import quantize_activation
    x = bf16_tensor(mxfp8_golden[case + "_x"], cuda)
    q, s = quantize_activation(x)
    assert np.array_equal(q.cpu().numpy(), mxfp8_golden[case + "_q"])
    assert np.array_equal(s.cpu().numpy(), mxfp8_golden[case + "_s"])


def test_device_quantiser_boundary_kat(cuda, mxfp8_golden):
    from vdn_b200.mxfp8_quant import launch_quantize
    x = torch.from_numpy(mxfp8_golden["kat_x"]).bfloat16()
    # The KAT is fp32-exact in bf16 except 1e-38 / -3e-39 (bf16 subnormal); compare
    # against the oracle on the bf16 values the device sees.
    q, s = launch_quantize(x.to(cuda))
    rq, rs = mx.quantize(x.float().numpy())
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)


@pytest.mark.parametrize("shape", [(0, 7), (1, 1), (17, 37), (129, 133), (128, 256), (300, 1000)])
def test_strided_rows_and_odd_shapes(cuda, shape):
    from vdn_b200.mxfp8_quant import quantize_activation, quantize_cpu
    m, k = shape
    g = torch.Generator().manual_seed(42)
    base = torch.randn(m * 2, k + 8, generator=g).bfloat16()
    x = base[::2, 3:3 + k]                      # non-contiguous rows, misaligned start
    q, s = quantize_activation(base.to(cuda)[::2, 3:3 + k])
    cq, cs = quantize_cpu(x)
    assert torch.equal(q.cpu(), cq) and torch.equal(s.cpu(), cs)


def test_subnormals_and_signed_zero(cuda):
    from vdn_b200.mxfp8_quant import launch_quantize
    vals = torch.tensor([1e-40, -2e-39, 0.0, -0.0, 3e-39, -1e-45, 5e-41, 1e-39] * 4)
    x = torch.stack([vals, -vals, vals * 1e30, torch.zeros_like(vals)]).bfloat16()
    q, s = launch_quantize(x.to(cuda))
    rq, rs = mx.quantize(x.float().numpy())
    assert np.array_equal(q.cpu().numpy(), rq) and np.array_equal(s.cpu().numpy(), rs)


@pytest.mark.parametrize("value", [float("nan"), float("inf")])
def test_reject_nonfinite_activation(cuda, value):
    from vdn_b200.mxfp8_quant import quantize_activation
    x = torch.ones(3, 64, dtype=torch.bfloat16, device=cuda)
    x[1, 40] = value
    with pytest.raises(ValueError, match="nonfinite MXFP8 activation"):
        quantize_activation(x)
    quantize_activation(x, check_finite=False)   # caller-owned guard: no raise


@pytest.mark.parametrize("rows,k", [(1, 128), (129, 256), (131, 1792), (129, 5120), (3, 200), (5, 12800)])
def test_producers_layout_rounding_and_finite(cuda, rows, k):
    from vdn_b200.mxfp8_kernels import (launch_gelu_quantize, launch_prenorm_quantize,
                                        launch_swiglu_quantize)
    from vdn_b200.mxfp8_quant import quantize_activation
    torch.manual_seed(429)
    x = torch.randn(rows * 2, 2 * k, device=cuda, dtype=torch.bfloat16)[::2]
    q, s, f = launch_swiglu_quantize(x)
    a, gt = x[:, :k].float(), x[:, k:].float()
    ref = (a * (gt * torch.sigmoid(gt))).bfloat16()
    qr, sr = quantize_activation(ref)
    # a * silu(g) may differ from torch's by one bf16 ulp (exp); compare decoded values.
    got = mx.dequantize(q.cpu().numpy(), s.cpu().numpy())[:rows, :k]
    want = mx.dequantize(qr.cpu().numpy(), sr.cpu().numpy())[:rows, :k]
    np.testing.assert_allclose(got, want, rtol=0.07, atol=1e-3)
    assert bool(f.all())
    for approx in ("tanh", "none"):
        up = x[:, :k]
        q, s, f = launch_gelu_quantize(up, approximate=approx)
        ref = torch.nn.functional.gelu(up.float(), approximate=approx).bfloat16()
        got = mx.dequantize(q.cpu().numpy(), s.cpu().numpy())[:rows, :k]
        np.testing.assert_allclose(got, ref.float().cpu().numpy(), rtol=0.07, atol=0.02)
        assert bool(f.all())
    hidden = x[:, :k]
    w = torch.randn(k, device=cuda, dtype=torch.bfloat16)
    scale, shift = torch.randn(7, k * 6, device=cuda, dtype=torch.bfloat16).chunk(6, -1)[:2]
    idx = torch.arange(rows, device=cuda) % 7
    y, q, s, f = launch_prenorm_quantize(hidden, w, 1e-6, scale, shift, idx, write_bf16=True)
    oracle = hidden.float() * torch.rsqrt(hidden.float().square().mean(-1, keepdim=True) + 1e-6) * w.float()
    oracle = (oracle * (1 + scale[idx].float()) + shift[idx].float()).bfloat16()
    torch.testing.assert_close(y, oracle, atol=.03125, rtol=.008)
    qr, sr = quantize_activation(y)
    assert torch.equal(q, qr) and torch.equal(s, sr) and bool(f.all())
    _, q2, s2, f2 = launch_prenorm_quantize(hidden, w, 1e-6, scale, shift, idx, write_bf16=False)
    assert torch.equal(q, q2) and torch.equal(s, s2) and bool(f2.all())
    x[0, 0] = float("nan")
    assert not bool(launch_swiglu_quantize(x)[2].all())
    assert not bool(launch_prenorm_quantize(x[:, :k], w, 1e-6, scale, shift, idx,
                                            write_bf16=False)[3].all())


def test_finite_parts_modes(cuda):
    from vdn_b200.mxfp8_kernels import finite_parts
    x = torch.ones(100000, device=cuda)
    assert bool(finite_parts(x).all())
    x[-1] = float("inf")
    parts = finite_parts(x)
    assert parts.numel() == 25 and not bool(parts[-1]) and bool(parts[:-1].all())
    assert not bool(finite_parts(torch.full((128,), 127, device=cuda, dtype=torch.uint8), 1).all())
    assert not bool(finite_parts(torch.full((4,), 255, device=cuda, dtype=torch.uint8), 2).all())
    assert bool(finite_parts(torch.full((4,), 254, device=cuda, dtype=torch.uint8), 2).all())
    assert bool(finite_parts(torch.ones(10, device=cuda, dtype=torch.bfloat16)).all())


def test_quantiser_full_size_properties(cuda):
    """BASELINE config-1 activation (32760 x 5120, 1% outlier channels x50):
    size-independent checks -- padding, scale bound and dequant round trip --
    plus a bit-exact slice against the oracle."""
    from vdn_b200.mxfp8_quant import quantize_activation
    g = torch.Generator(device=cuda).manual_seed(7)
    x = torch.randn(32760, 5120, device=cuda, generator=g)
    idx = torch.randperm(5120, device=cuda, generator=g)[:51]
    x[:, idx] *= 50
    x = x.bfloat16()
    q, s = quantize_activation(x)
    assert q.shape == (32768, 5120) and s.numel() == 32768 * 160
    assert int(q[32760:].count_nonzero()) == 0
    rows = slice(12800, 13056)
    rq, rs = mx.quantize(x[rows].float().cpu().numpy())
    assert np.array_equal(q[rows].cpu().numpy(), rq[:256])
    scales = mx.unswizzle(s.cpu().numpy(), 32768, 5120)
    assert np.array_equal(scales[rows], mx.unswizzle(rs, 256, 5120))
    back = torch.from_numpy(mx.dequantize(q[:4096].cpu().numpy(), mx.swizzle(scales[:4096])))
    torch.testing.assert_close(back[:4096].float(), x[:4096].float().cpu(), rtol=.063, atol=.001 * 50)


@pytest.mark.parametrize("d,hl", [(128, 3), (64, 2)])
def test_quantize_scatter_routes_to_owners(cuda, d, hl):
    """vdn_mxfp8_quantize_scatter: a head-sharded [T, hl, d] output lands, as MXFP8,
    in each owner's padded operand exactly as quantize_activation of the owner's
    rows of the full [T, H*d] matrix (three emulated owners with ragged rows)."""
    import ctypes as C
    from vdn_b200 import _lib
    from vdn_b200.mxfp8_quant import quantize_activation
    T, H = 300, 2 * hl
    head0 = hl                            # this "rank" holds heads [hl, 2 hl)
    full = torch.randn(T, H, d, device=cuda).bfloat16()
    src = full[:, head0:head0 + hl]       # strided view [T, hl, d]
    starts = [0, 130, 250, 300]
    kp = H * d
    owners = []
    for p in range(3):
        rp = (starts[p + 1] - starts[p] + 127) // 128 * 128
        owners.append((torch.zeros(rp, kp, dtype=torch.uint8, device=cuda),
                       torch.zeros(rp * kp // 32, dtype=torch.uint8, device=cuda)))
    _lib.call("vdn_mxfp8_quantize_scatter", _lib.ptr(src), T, hl, d, src.stride(0), src.stride(1), head0,
              kp, 3, (C.c_int64 * 4)(*starts), (C.c_void_p * 3)(*[o[0].data_ptr() for o in owners]),
              (C.c_void_p * 3)(*[o[1].data_ptr() for o in owners]), None, _lib.stream_of(cuda))
    torch.cuda.synchronize()
    cols = slice(head0 * d, (head0 + hl) * d)
    for p in range(3):
        rows = full[starts[p]:starts[p + 1]].reshape(-1, kp)
        masked = torch.zeros_like(rows)
        masked[:, cols] = rows[:, cols]
        q, s = quantize_activation(masked)
        assert torch.equal(owners[p][0][:, cols], q[:, cols]), p
        # scale bytes of this rank's column blocks only (others stay untouched)
        r = torch.arange(q.shape[0], device=cuda)[:, None]
        c = torch.arange(kp // 32, device=cuda)[None, :]
        idx = ((r // 128) * (kp // 128) + c // 4) * 512 + r % 32 * 16 + (r % 128 // 32) * 4 + c % 4
        blk = slice(head0 * d // 32, (head0 + hl) * d // 32)
        assert torch.equal(owners[p][1][idx[:, blk]], s[idx[:, blk]]), p
