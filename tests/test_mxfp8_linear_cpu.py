"""CPU: the MXFP8 linear API around the GEMM (reference src/models/ops/mxfp8_linear.py).

convert_linear_to_mxfp8 (:145-180): off by default, the seven roles of every block,
records, refusals (training mode, a non-Linear role, a role off the CPU/meta
devices, tied weights) raised before anything is replaced, meta models.  The
projection helpers (:105-124): projection_features, project, project_to_out with a
(projection, dropout) pair.  MXFP8Linear construction (:36-58): buffers, no
.weight, bias kept, argument checks.  The reference's own tests pin the same
behaviour (tests/test_paper_stack_mxfp8_ops.py).
"""
import numpy as np
import pytest
import torch
from torch import nn

from oracle import mxfp8 as omx
from vdn_b200.mxfp8_linear import (SUPPORTED_ROLES, MXFP8Linear, convert_linear_to_mxfp8,
                                   project, project_to_out, projection_features)


class _Attn(nn.Module):
    def __init__(self, hd):
        super().__init__()
        self.orig = nn.Module()
        self.orig.to_q, self.orig.to_k, self.orig.to_v = (nn.Linear(hd, hd) for _ in range(3))
        self.orig.to_out = nn.ModuleList([nn.Linear(hd, hd), nn.Dropout(0.0)])
        self.to_out_linear = nn.Linear(hd, hd, bias=False)
        self.norm = nn.LayerNorm(hd)


class _FF(nn.Module):
    def __init__(self, hd, ffn):
        super().__init__()
        self.net = nn.ModuleList([nn.Module(), nn.GELU(), nn.Linear(ffn, hd)])
        self.net[0].proj = nn.Linear(hd, ffn)


class _Block(nn.Module):
    def __init__(self, hd=64, ffn=96):
        super().__init__()
        self.attn, self.ff = _Attn(hd), _FF(hd, ffn)


class _Model(nn.Module):
    def __init__(self, blocks=2, device=None):
        super().__init__()
        with torch.device(device or "cpu"):
            self.transformer_blocks = nn.ModuleList(_Block() for _ in range(blocks))
            self.proj_out = nn.Linear(64, 64)


def test_disabled_returns_empty_and_changes_nothing():
    m = _Model().eval()
    before = {n: type(x) for n, x in m.named_modules()}
    assert convert_linear_to_mxfp8(m) == []
    assert convert_linear_to_mxfp8(m, enabled=False) == []
    assert {n: type(x) for n, x in m.named_modules()} == before


def test_converts_all_seven_roles_of_every_block():
    torch.manual_seed(0)
    m = _Model(blocks=2).eval()
    want = {(i, r): m.transformer_blocks[i].get_submodule(p).weight.detach().clone()
            for i in range(2) for r, p in SUPPORTED_ROLES.items()}
    recs = convert_linear_to_mxfp8(m, enabled=True)
    assert [(r["block"], r["role"]) for r in recs] == [(i, r) for i in range(2) for r in SUPPORTED_ROLES]
    assert recs[3]["module"] == "transformer_blocks.0.attn.orig.to_out.0"
    assert (recs[5]["in_features"], recs[5]["out_features"]) == (64, 96)
    for i, block in enumerate(m.transformer_blocks):
        for role, path in SUPPORTED_ROLES.items():
            mod = block.get_submodule(path)
            assert type(mod) is MXFP8Linear and not hasattr(mod, "weight")
            q, s = omx.quantize(want[(i, role)].float().numpy())
            assert np.array_equal(mod.weight_data.numpy(), q) and np.array_equal(mod.weight_scale.numpy(), s)
    # The roots, norms and the dropout half of to_out stay untouched.
    assert type(m.proj_out) is nn.Linear and type(m.transformer_blocks[0].attn.norm) is nn.LayerNorm
    assert type(m.transformer_blocks[0].attn.orig.to_out[1]) is nn.Dropout
    assert m.transformer_blocks[0].attn.to_out_linear.bias is None
    assert m.transformer_blocks[0].attn.orig.to_q.bias is not None


def test_refuses_training_mode():
    with pytest.raises(ValueError, match="convert an eval model"):
        convert_linear_to_mxfp8(_Model().train(), enabled=True)


def test_refuses_bad_flags():
    with pytest.raises(ValueError, match="booleans"):
        convert_linear_to_mxfp8(_Model().eval(), enabled=1)
    with pytest.raises(ValueError, match="booleans"):
        convert_linear_to_mxfp8(_Model().eval(), enabled=True, check_finite="yes")


def test_tied_weights_refused_before_any_change():
    m = _Model().eval()
    b = m.transformer_blocks[1]
    b.ff.net[2].weight = m.transformer_blocks[0].ff.net[2].weight      # tied across blocks
    with pytest.raises(ValueError, match="tied MXFP8 target weights are unsupported"):
        convert_linear_to_mxfp8(m, enabled=True)
    assert all(type(x) is not MXFP8Linear for x in m.modules())
    m2 = _Model().eval()
    m2.proj_out.weight = m2.transformer_blocks[0].attn.orig.to_q.weight  # tied to a non-target
    with pytest.raises(ValueError, match="tied"):
        convert_linear_to_mxfp8(m2, enabled=True)


def test_non_linear_role_refused():
    m = _Model().eval()
    m.transformer_blocks[1].attn.to_out_linear = nn.Identity()
    with pytest.raises(ValueError, match="1:linear_out requires a merged CPU/meta nn.Linear"):
        convert_linear_to_mxfp8(m, enabled=True)
    assert all(type(x) is not MXFP8Linear for x in m.modules())


def test_meta_model_converts_shapes_only():
    m = _Model(blocks=1, device="meta").eval()
    recs = convert_linear_to_mxfp8(m, enabled=True)
    assert len(recs) == 7
    up = m.transformer_blocks[0].ff.net[0].proj
    assert up.weight_data.is_meta and tuple(up.weight_data.shape) == (128, 128)
    assert tuple(up.weight_scale.shape) == (128 * 128 // 32,)


def test_mxfp8linear_construction_checks():
    lin = nn.Linear(40, 24)
    with pytest.raises(ValueError, match="check_finite must be a bool"):
        MXFP8Linear(lin, check_finite=0)
    with pytest.raises(TypeError, match="ordinary merged nn.Linear"):
        MXFP8Linear(nn.Bilinear(4, 4, 4))
    with torch.no_grad():
        lin.bias[3] = float("nan")
    with pytest.raises(ValueError, match="nonfinite"):
        MXFP8Linear(lin)
    m = MXFP8Linear(nn.Linear(40, 24))
    assert tuple(m.weight_data.shape) == (128, 128) and m.weight_data.dtype == torch.uint8
    assert tuple(m.weight_scale.shape) == (512,) and not m.training
    assert not m.bias.requires_grad
    with pytest.raises(ValueError, match="eval BF16 output only"):
        m.forward_quantized(torch.zeros(128, 128, dtype=torch.uint8), torch.zeros(512, dtype=torch.uint8),
                            out_dtype=torch.float32)


def test_projection_helpers():
    lin = nn.Linear(8, 6)
    x = torch.randn(3, 8)
    assert projection_features(lin) == (8, 6)
    assert projection_features(MXFP8Linear(nn.Linear(40, 24))) == (40, 24)
    with pytest.raises(TypeError, match="unsupported projection module"):
        projection_features(nn.Conv1d(2, 2, 1))
    torch.testing.assert_close(project(lin, x), lin(x))
    drop = nn.Dropout(0.0)
    torch.testing.assert_close(project_to_out(nn.ModuleList([lin, drop]), x), lin(x))
    torch.testing.assert_close(project_to_out([lin, drop], x), lin(x))
    torch.testing.assert_close(project_to_out(lin, x), lin(x))
    with pytest.raises(ValueError, match="expected projection/dropout pair"):
        project_to_out(nn.Sequential(lin, drop, drop), x)
    with pytest.raises(TypeError):
        project_to_out([nn.Conv1d(2, 2, 1), drop], x)
