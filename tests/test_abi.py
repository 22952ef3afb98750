"""CPU: the C-ABI library loads, exports every declared symbol, and the host-side
logic (native host quantiser, argument validation, API checks) behaves like the
reference's CPU contracts (tests/test_paper_stack_mxfp8_ops.py:49-83)."""
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from vdn_b200 import _lib
from vdn_b200.mxfp8_quant import padded_shape, quantize_cpu, scale_numel, swizzle_scales
from oracle import mxfp8 as mx
from helpers import bf16_tensor

HEADER = Path(__file__).resolve().parents[1] / "include" / "vdn_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(vdn_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), set(names) ^ set(_lib.SIGNATURES)
    assert lib.vdn_abi_version() == 1


def test_padded_shape_matches_native():
    rp, kp = _lib.C.c_int64(), _lib.C.c_int64()
    for rows, k in [(0, 1), (1, 1), (129, 129), (32760, 5120), (32760, 13824)]:
        _lib.call("vdn_mxfp8_padded_shape", rows, k, _lib.C.byref(rp), _lib.C.byref(kp))
        assert (rp.value, kp.value) == padded_shape(rows, k) == mx.padded_shape(rows, k)
        assert scale_numel(rows, k) == mx.scale_numel(rows, k)
    with pytest.raises(ValueError):
        _lib.call("vdn_mxfp8_padded_shape", 4, 0, _lib.C.byref(rp), _lib.C.byref(kp))


@pytest.mark.parametrize("case", ["cfg0", "outlier", "kat"] + [f"shape{i}" for i in range(6)])
def test_native_host_quantiser_bit_exact_vs_reference(mxfp8_golden, case):
    raw = mxfp8_golden[case + "_x"]
    x = bf16_tensor(raw) if raw.dtype == np.uint16 else torch.from_numpy(raw)
    before = x.clone()
    q, s = quantize_cpu(x, chunk_rows=7)
    assert torch.equal(x, before)
    assert np.array_equal(q.numpy(), mxfp8_golden[case + "_q"])
    assert np.array_equal(s.numpy(), mxfp8_golden[case + "_s"])


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_native_host_quantiser_dtypes_and_strides(dtype):
    g = torch.Generator().manual_seed(3)
    base = (torch.randn(70, 400, generator=g) * 3).to(dtype)
    x = base[::2, 5:305]
    q, s = quantize_cpu(x)
    rq, rs = mx.quantize(x.float().numpy())
    assert np.array_equal(q.numpy(), rq) and np.array_equal(s.numpy(), rs)


def test_host_quantiser_subnormal_fp16():
    x = torch.tensor([[6e-8, -6e-8, 1e-5, 0.0] * 8], dtype=torch.float16)
    q, s = quantize_cpu(x)
    rq, rs = mx.quantize(x.float().numpy())
    assert np.array_equal(q.numpy(), rq) and np.array_equal(s.numpy(), rs)


@pytest.mark.parametrize("value", [float("nan"), float("inf"), -float("inf")])
def test_reject_nonfinite_cpu(value):
    with pytest.raises(ValueError, match="nonfinite"):
        quantize_cpu(torch.tensor([[value]]))


def test_cpu_quantiser_contracts():
    with pytest.raises(ValueError, match="floating 2D"):
        quantize_cpu(torch.zeros(3, dtype=torch.float32))
    with pytest.raises(ValueError, match="chunk_rows"):
        quantize_cpu(torch.zeros(2, 2), chunk_rows=0)
    q, s = quantize_cpu(torch.zeros(0, 5))
    assert q.shape == (0, 128) and s.numel() == 0
    q, s = quantize_cpu(torch.empty(300, 70, device="meta"))
    assert q.shape == (384, 128) and s.shape == (384 * 4,) and q.is_meta


def test_swizzle_scales_matches_oracle():
    natural = (torch.arange(256 * 12) % 251).to(torch.uint8).reshape(256, 12)
    assert np.array_equal(swizzle_scales(natural).numpy(), mx.swizzle(natural.numpy()))


def test_cpu_tensors_rejected_before_launch():
    from vdn_b200.mxfp8_quant import quantize_activation
    from vdn_b200.paper_factor import paper_delta_factors
    with pytest.raises(ValueError, match="CUDA BF16"):
        quantize_activation(torch.zeros(2, 32, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        paper_delta_factors(torch.zeros(128, 128), torch.zeros(128, 128))
    with pytest.raises(TypeError):
        paper_delta_factors(None, torch.zeros(128, 128))
    with pytest.raises(TypeError):
        paper_delta_factors(torch.zeros(128, 128, dtype=torch.float64), torch.zeros(128, 128))


def test_branch_module_contracts():
    from vdn_b200.linear_attention import BidirectionalLinearBranch, window_bounds
    with pytest.raises(ValueError):
        BidirectionalLinearBranch(16, 2, 128, delta_rule="sana_scaled")
    with pytest.raises(ValueError):
        BidirectionalLinearBranch(16, 2, 128, short_conv=("k", "k"))
    with pytest.raises(ValueError):
        BidirectionalLinearBranch(16, 2, 128, short_conv=("x",))
    conv = BidirectionalLinearBranch(16, 2, 128, short_conv=("k", "v"))
    assert {"short_conv.k_sp.weight", "short_conv.k_tm.weight", "short_conv.v_sp.weight",
            "short_conv.v_tm.weight"} <= set(dict(conv.named_parameters()))
    assert conv.short_conv.k_sp.weight.shape == (256, 1, 5, 5)
    assert conv.short_conv.k_tm.weight.shape == (256, 1, 5)
    b = BidirectionalLinearBranch(16, 2, 128)
    names = set(dict(b.named_parameters()))
    assert {"alpha.A_log", "alpha.dt_bias", "alpha.down.weight", "alpha.up.weight",
            "beta_proj.weight", "output_gate.down.weight", "output_gate.up.weight",
            "output_gate.up.bias", "norm.weight"} == names
    raw = (torch.zeros(4, 2, 128, dtype=torch.bfloat16),) * 3
    with torch.no_grad(), pytest.raises(ValueError, match="CUDA BF16"):
        b(torch.zeros(4, 16), 1, 4, window_bounds(1, 1), raw)
    with pytest.raises(RuntimeError, match="no_grad"):
        b(torch.zeros(4, 16), 1, 4, window_bounds(1, 1), raw)
