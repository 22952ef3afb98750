"""Short conv: the oracle against the reference fixtures (CPU), and the kernel against
the oracle and the reference features (GPU).

tests/golden/sepconv_golden.npz holds the reference LinearAttentionSepConv run on CPU
(features.py:133-209): spatial half, eager temporal shift, activated features.
"""
import numpy as np
import pytest
import torch

from oracle import sepconv as osc
from oracle.mxfp8 import bf16_to_f32


@pytest.fixture(scope="module")
def golden():
    from pathlib import Path
    return np.load(Path(__file__).parent / "golden" / "sepconv_golden.npz")


def _case(z, name, proj):
    f, gh, gw, h, d = (int(v) for v in z[f"{name}_geom"])
    key = f"{name}_{proj}"
    x = bf16_to_f32(z[f"{key}_x"]).reshape(f * gh * gw, h, d)
    wsp = bf16_to_f32(z[f"{key}_wsp"]).reshape(h * d, 25)
    wtm = bf16_to_f32(z[f"{key}_wtm"]).reshape(h * d, 5)
    return (f, gh, gw, h, d), x, wsp, wtm, key


@pytest.mark.parametrize("name", ["small", "d128"])
@pytest.mark.parametrize("proj", ["k", "v"])
def test_oracle_pinned_to_reference(golden, name, proj):
    (f, gh, gw, h, d), x, wsp, wtm, key = _case(golden, name, proj)
    sp = osc.spatial(x.reshape(-1, h * d), wsp, f, (gh, gw))
    assert np.array_equal(sp.ravel(), bf16_to_f32(golden[f"{key}_spatial"]).ravel())
    tm = osc.temporal_eager(sp, wtm)
    assert np.array_equal(tm.ravel(), bf16_to_f32(golden[f"{key}_temporal"]).ravel())
    feat = osc.conv_features(x, wsp, wtm, f, (gh, gw), proj != "v", eager=True)
    assert np.array_equal(feat.ravel(), bf16_to_f32(golden[f"{key}_features"]).ravel())
    # The fused temporal form (one rounding) stays close to the eager chain (per-op
    # roundings): a few bf16 ulps of the terms' magnitude, even where the taps cancel.
    fused = osc.temporal(sp, wtm)
    terms = np.abs(sp).mean()
    assert np.max(np.abs(fused - tm)) <= 2 ** -5 * terms * 4
    assert np.linalg.norm(fused - tm) / np.linalg.norm(tm) < 5e-3


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["small", "d128"])
@pytest.mark.parametrize("proj", ["k", "v"])
def test_kernel_matches_oracle_and_reference(cuda, golden, name, proj):
    from vdn_b200.short_conv import sepconv
    (f, gh, gw, h, d), x, wsp, wtm, key = _case(golden, name, proj)
    xt = torch.from_numpy(x).bfloat16().to(cuda)
    out = sepconv(xt, f, (gh, gw), torch.from_numpy(wsp).to(cuda), torch.from_numpy(wtm).to(cuda))
    torch.cuda.synchronize()
    got = out.float().cpu().numpy().reshape(f, gh * gw, h * d)
    sp = osc.spatial(x.reshape(-1, h * d), wsp, f, (gh, gw))
    want = osc.temporal(sp, wtm)
    # fp32 accumulation of the spatial taps vs the exact sum: rare one-ulp flips.
    mism = np.mean(got != want)
    assert mism < 0.02, mism
    rel = np.linalg.norm(got - want) / np.linalg.norm(want)
    assert rel < 2e-3, rel
    ref_tm = bf16_to_f32(golden[f"{key}_temporal"]).reshape(got.shape)
    assert np.linalg.norm(got - ref_tm) / np.linalg.norm(ref_tm) < 5e-3


@pytest.mark.gpu
def test_kernel_strided_rows_and_head_slice(cuda):
    """Rows with a stride (a view of a wider QKV buffer) and a head slice of the weights."""
    from vdn_b200.short_conv import LinearAttentionSepConv
    torch.manual_seed(5)
    f, gh, gw, H, d = 3, 4, 6, 4, 64
    conv = LinearAttentionSepConv(H * d, ("k",)).to(cuda).to(torch.bfloat16)
    wide = torch.randn(f * gh * gw, 3 * H * d, device=cuda).bfloat16()
    k = wide[:, H * d:2 * H * d].view(-1, H, d)
    full = conv.apply("k", k, f, (gh, gw))
    part = conv.apply("k", k[:, 1:3], f, (gh, gw), heads=slice(1, 3))
    torch.cuda.synchronize()
    assert torch.equal(part, full[:, 1:3])
    assert conv.apply("q", k, f, (gh, gw)) is k


@pytest.mark.gpu
@torch.no_grad()
def test_branch_with_short_conv_matches_oracle(cuda):
    """BidirectionalLinearBranch(short_conv=("k", "v")) == the oracle body on the
    conv outputs (features.py:187-209 + branch.py:404-482), relative L2 < 4e-3."""
    from oracle import vda as ovda
    from vdn_b200.linear_attention import BidirectionalLinearBranch, window_bounds
    torch.manual_seed(7)
    f, gh, gw, H, d = 5, 4, 6, 2, 128
    s = gh * gw
    n = f * s
    br = BidirectionalLinearBranch(64, H, d, short_conv=("k", "v")).to(cuda)
    br.short_conv.to(torch.bfloat16)
    q, k, v = (torch.randn(n, H, d, device=cuda).bfloat16() for _ in range(3))
    beta = torch.sigmoid(torch.randn(n, H, device=cuda)).bfloat16()
    gate = torch.rand(n, H, d, device=cuda).bfloat16()
    fm = torch.randn(f, 64, device=cuda)
    bounds = window_bounds(f, 1)
    out = br(None, f, s, bounds, (q, k, v), frame_size=(gh, gw), heads=slice(0, H), beta=beta,
             gate=gate, frame_mean=fm)
    torch.cuda.synchronize()
    alpha = br.alpha(fm).float().cpu().numpy()

    def conv_np(t, proj):
        w_sp = getattr(br.short_conv, f"{proj}_sp").weight.float().cpu().numpy().reshape(H * d, 25)
        w_tm = getattr(br.short_conv, f"{proj}_tm").weight.float().cpu().numpy().reshape(H * d, 5)
        sp = osc.spatial(t.float().cpu().numpy().reshape(n, H * d), w_sp, f, (gh, gw))
        return osc.temporal(sp, w_tm).reshape(n, H, d)

    ref = ovda.readout(q.float().cpu().numpy(), conv_np(k, "k"), conv_np(v, "v"),
                       beta.float().cpu().numpy(), gate.float().cpu().numpy(), alpha, bounds, f, s)
    got = out.float().cpu().numpy()
    err = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert err < 4e-3, err
