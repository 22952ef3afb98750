"""GPU: the VDA stage kernels and the full branch against the reference fixtures and
the oracle, mirroring the reference's GPU oracles (tests/test_paper_stack_vda_ops.py,
tests/test_paper_stack_vda_factor.py).

Tolerances (bf16 outputs): relative L2 < 4e-3 and max-abs <= 0.0625 against the
reference's own eager branch output -- the reference's own paper-vs-fp64 test
allows relative L2 0.004 (test_paper_stack_vda_ops.py:256).  fp32 stages use the
reference's limits: factors rel-L2 1e-5 / 3e-5, scans atol 3e-6 rtol 3e-5.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import mxfp8 as mx
from oracle import vda as ovda
from helpers import bf16_tensor, rel_l2, max_abs

pytestmark = pytest.mark.gpu
VDA_CASES = ["cfg0", "d128", "d128_text", "d128_anchor", "d128_wide"]


def _case(g, name, dev):
    f, s, h, d, skip, tl = (int(x) for x in g[name + "_geometry"])
    t = lambda k: bf16_tensor(g[name + "_" + k], dev)
    rec = dict(f=f, s=s, h=h, d=d, skip=bool(skip), tl=tl, q=t("q"), k=t("k"), v=t("v"),
               beta=t("beta"), gate=t("gate"), alpha=torch.from_numpy(g[name + "_alpha"]).to(dev),
               bounds=[tuple(int(v) for v in x) for x in g[name + "_bounds"]],
               out=mx.bf16_to_f32(g[name + "_out"]))
    if tl:
        rec.update(tk=t("tk"), tv=t("tv"), tbeta=t("tbeta"))
    return rec


@pytest.mark.parametrize("case", VDA_CASES)
@torch.no_grad()
def test_branch_matches_reference_eager_body(cuda, vda_golden, case):
    from vdn_b200.linear_attention import BidirectionalLinearBranch
    c = _case(vda_golden, case, cuda)
    branch = BidirectionalLinearBranch(16, c["h"], c["d"]).to(cuda)
    alpha = c["alpha"]
    branch.alpha.forward = lambda fm, heads=None: alpha[1:-1] if fm.shape[0] == c["f"] - 2 else alpha
    text = {}
    if c["tl"]:
        tq = torch.zeros_like(c["tk"])
        text = dict(text_qkv_raw=(tq, c["tk"], c["tv"]), text_beta=c["tbeta"])
    out = branch(None, c["f"], c["s"], c["bounds"], (c["q"], c["k"], c["v"]), skip_ends=c["skip"],
                 heads=slice(0, c["h"]), beta=c["beta"], gate=c["gate"],
                 frame_mean=torch.zeros(c["f"], 16, device=cuda), **text)
    got = out.float().cpu().numpy()
    assert out.dtype == torch.bfloat16 and out.shape == (c["f"] * c["s"], c["h"] * c["d"])
    assert rel_l2(got, c["out"]) < 4e-3, rel_l2(got, c["out"])
    assert max_abs(got, c["out"]) <= 0.0625
    if c["skip"]:
        assert not bool(out[:c["s"]].count_nonzero()) and not bool(out[-c["s"]:].count_nonzero())


@torch.no_grad()
def test_statistics_vs_reference_stages(cuda, vda_stages_golden):
    from vdn_b200.linear_attention import vda_statistics
    g = vda_stages_golden
    k, v, beta = (bf16_tensor(g[n], cuda) for n in ("k", "v", "beta"))
    a, b = vda_statistics(k, v, beta, features_applied=True)
    assert rel_l2(a.cpu().numpy(), g["a"]) < 5e-7
    assert rel_l2(b.cpu().numpy(), g["b"]) < 1e-4
    torch.testing.assert_close(a, a.transpose(-1, -2), atol=2e-6, rtol=1e-6)


@pytest.mark.parametrize("s", [1, 33, 129, 1008])
@torch.no_grad()
def test_statistics_raw_features_vs_oracle(cuda, s):
    from vdn_b200.linear_attention import vda_statistics
    g = torch.Generator(device="cpu").manual_seed(s)
    raw_k = torch.randn(3, s, 2, 128, generator=g).bfloat16()   # [F, S, H, d] token-major
    raw_v = torch.randn(3, s, 2, 128, generator=g).bfloat16()
    beta = torch.rand(3, s, 2, generator=g).bfloat16()
    a, b = vda_statistics(raw_k.to(cuda).permute(0, 2, 1, 3), raw_v.to(cuda).permute(0, 2, 1, 3),
                          beta.to(cuda).permute(0, 2, 1), features_applied=False)
    kf = ovda.features(raw_k.float().numpy(), True).transpose(0, 2, 1, 3)
    vf = ovda.features(raw_v.float().numpy(), False).transpose(0, 2, 1, 3)
    oa, ob = ovda.frame_statistics(kf, vf, beta.float().numpy().transpose(0, 2, 1))
    # Features may differ from the eager rounding by one bf16 ulp.
    assert rel_l2(a.cpu().numpy(), oa) < 2e-3
    assert rel_l2(b.cpu().numpy(), ob) < 4e-3


@torch.no_grad()
def test_statistics_raw_features_extreme_inputs(cuda):
    """SiLU inputs far below zero (the kernel raises them to -43.5 on the packed bf16
    pair, where |silu| < 6e-18 either way) and large positive ones: A and B still
    match the oracle, with no inf or NaN."""
    from vdn_b200.linear_attention import vda_statistics
    g = torch.Generator(device="cpu").manual_seed(3)
    raw_k = torch.randn(2, 96, 2, 128, generator=g)
    raw_v = torch.randn(2, 96, 2, 128, generator=g)
    mask = torch.rand(raw_k.shape, generator=g) < 0.05
    raw_k[mask] = -90.0
    raw_v[mask] = -300.0
    raw_k[..., 5] = 60.0
    raw_v[..., 7] = -1e4
    raw_k, raw_v = raw_k.bfloat16(), raw_v.bfloat16()
    beta = torch.rand(2, 96, 2, generator=g).bfloat16()
    a, b = vda_statistics(raw_k.to(cuda).permute(0, 2, 1, 3), raw_v.to(cuda).permute(0, 2, 1, 3),
                          beta.to(cuda).permute(0, 2, 1), features_applied=False)
    assert bool(torch.isfinite(a).all()) and bool(torch.isfinite(b).all())
    kf = ovda.features(raw_k.float().numpy(), True).transpose(0, 2, 1, 3)
    vf = ovda.features(raw_v.float().numpy(), False).transpose(0, 2, 1, 3)
    oa, ob = ovda.frame_statistics(kf, vf, beta.float().numpy().transpose(0, 2, 1))
    assert rel_l2(a.cpu().numpy(), oa) < 2e-3
    assert rel_l2(b.cpu().numpy(), ob) < 4e-3


def _stats_inputs(frames, heads, tokens, beta_scale=1.0, seed=0, d=128):
    g = torch.Generator(device="cpu").manual_seed(seed)
    shape = (frames, heads, tokens, d)
    k = F.normalize(F.silu(torch.randn(shape, generator=g)), dim=-1)
    v = F.silu(torch.randn(shape, generator=g))
    beta = torch.sigmoid(torch.randn(shape[:-1], generator=g)) * beta_scale
    alpha = torch.rand(frames, heads, d, generator=g) * 0.9 + 0.1
    A = (k * beta.unsqueeze(-1)).transpose(-1, -2) @ k
    A = 0.5 * (A + A.transpose(-1, -2))
    B = (v * beta.unsqueeze(-1)).transpose(-1, -2) @ k
    return A.float().contiguous(), B.float().contiguous(), alpha.float().contiguous()


def _fp64_factors(A, B, alpha=None):
    a, b = A.double(), B.double()
    eye = torch.eye(a.shape[-1], dtype=torch.float64)
    system = eye + a
    rhs = eye.expand_as(a) if alpha is None else torch.diag_embed(alpha.double())
    t = torch.linalg.solve(system.transpose(-1, -2), rhs.transpose(-1, -2)).transpose(-1, -2)
    j = torch.linalg.solve(system.transpose(-1, -2), b.transpose(-1, -2)).transpose(-1, -2)
    return t, j


@pytest.mark.parametrize("frames,heads,tokens", [(1, 1, 16), (5, 3, 64), (11, 7, 1008)])
@pytest.mark.parametrize("beta_scale", [1.0, 50.0])
@pytest.mark.parametrize("with_alpha", [False, True])
@pytest.mark.parametrize("d", [64, 128])
def test_factors_vs_fp64(cuda, frames, heads, tokens, beta_scale, with_alpha, d):
    from vdn_b200.paper_factor import paper_delta_factors
    A, B, alpha = _stats_inputs(frames, heads, tokens, beta_scale, d=d)
    if not with_alpha:
        alpha = None
    ref = _fp64_factors(A, B, alpha)
    out = paper_delta_factors(A.to(cuda), B.to(cuda), None if alpha is None else alpha.to(cuda))
    for got, want, lim in zip(out, ref, (1e-5, 3e-5)):
        assert got.dtype == torch.float32 and torch.isfinite(got).all()
        assert rel_l2(got.double().cpu().numpy(), want.numpy()) < lim


def test_factors_stage_golden_and_inplace_semantics(cuda, vda_stages_golden):
    from vdn_b200.paper_factor import paper_delta_factors
    g = vda_stages_golden
    A, B, alpha = (torch.from_numpy(g[n]).to(cuda) for n in ("a", "b", "alpha"))
    snap = [x.clone() for x in (A, B, alpha)]
    t, j = paper_delta_factors(A, B, alpha)
    assert rel_l2(t.cpu().numpy(), g["t"]) < 1e-5 and rel_l2(j.cpu().numpy(), g["j"]) < 3e-5
    for x, y in zip((A, B, alpha), snap):
        assert torch.equal(x, y)
    # Storage offsets (misaligned contiguous views) give bit-identical results.
    store = torch.empty(A.numel() + 1, device=cuda)
    A1 = store[1:].view(A.shape)
    A1.copy_(A)
    t1, j1 = paper_delta_factors(A1, B, alpha)
    assert torch.equal(t1, t) and torch.equal(j1, j)
    e = torch.empty(0, 128, 128, device=cuda)
    assert all(x.numel() == 0 for x in paper_delta_factors(e, e))


@pytest.mark.parametrize("frames", [1, 2, 11, 31])
@pytest.mark.parametrize("text", [False, True])
@pytest.mark.parametrize("decay", [1.0, 0.7, 0.001])
def test_scan_and_gather_vs_fp64(cuda, frames, text, decay):
    from vdn_b200.linear_attention import vda_gather, vda_scan
    from vdn_b200.paper_factor import paper_delta_factors
    torch.manual_seed(frames)
    h, d = 2, 128
    k = F.normalize(torch.randn(frames, h, 9, d), dim=-1)
    a = (k.transpose(-1, -2) @ k).contiguous()
    b = torch.randn_like(a) * 0.1
    alpha = (torch.rand(frames, h, d) * 0.1 + 0.9) * decay
    t, inj = paper_delta_factors(a.to(cuda), b.to(cuda), alpha.to(cuda))
    seed = torch.randn(h, d, d) * .3 if text else None
    prefix, suffix = vda_scan(t, inj, None if seed is None else seed.to(cuda))
    op, osf = ovda.run_scans(t.double().cpu().numpy(), inj.double().cpu().numpy(),
                             None if seed is None else seed.double().numpy())
    torch.testing.assert_close(prefix.double().cpu(), torch.from_numpy(op), atol=3e-6, rtol=3e-5)
    torch.testing.assert_close(suffix.double().cpu(), torch.from_numpy(osf), atol=3e-6, rtol=3e-5)
    bounds = [(f - 2, f + 1) for f in range(frames)]
    for bridge in (True, False):
        got = vda_gather(prefix, suffix, alpha.to(cuda), bounds,
                         None if seed is None else seed.to(cuda), torch.float32, bridge)
        want = ovda.gather(op, osf, alpha.numpy(), bounds,
                           None if seed is None else seed.double().numpy(), bridge)
        torch.testing.assert_close(got.double().cpu(), torch.from_numpy(want), atol=4e-6, rtol=5e-5)


@pytest.mark.parametrize("heads,d", [(40, 128), (20, 128), (3, 128), (80, 64), (5, 64)])
def test_scan_row_blocking_vs_fp64(cuda, heads, d):
    """The scan picks 64, 32 or 16 state rows per CTA from the head count; every
    blocking gives the fp64 recurrence (seeded, 5 frames, both directions)."""
    from vdn_b200.linear_attention import vda_scan
    g = torch.Generator().manual_seed(heads * 7 + d)
    frames = 5
    t = (torch.randn(frames, heads, d, d, generator=g) * (0.9 / d ** 0.5)).to(cuda)
    inj = (torch.randn(frames, heads, d, d, generator=g) * 0.1).to(cuda)
    seed = torch.randn(heads, d, d, generator=g) * .3
    prefix, suffix = vda_scan(t, inj, seed.to(cuda))
    op, osf = ovda.run_scans(t.double().cpu().numpy(), inj.double().cpu().numpy(), seed.double().numpy())
    torch.testing.assert_close(prefix.double().cpu(), torch.from_numpy(op), atol=3e-6, rtol=3e-5)
    torch.testing.assert_close(suffix.double().cpu(), torch.from_numpy(osf), atol=3e-6, rtol=3e-5)


@torch.no_grad()
def test_gather_vs_reference_stages(cuda, vda_stages_golden):
    from vdn_b200.linear_attention import vda_gather
    g = vda_stages_golden
    pre, suf, alpha, seed = (torch.from_numpy(g[n]).to(cuda) for n in ("prefix", "suffix", "alpha", "seed"))
    bounds = [tuple(int(v) for v in x) for x in g["bounds"]]
    got = vda_gather(pre, suf, alpha, bounds, seed, torch.float32)
    assert rel_l2(got.cpu().numpy(), g["gathered"]) < 1e-6
    got0 = vda_gather(pre, suf, alpha, bounds, None, torch.float32)
    assert rel_l2(got0.cpu().numpy(), g["gathered_noseed"]) < 1e-6


def test_long_recurrence_102_frames(cuda):
    """Non-commuting transitions near identity over many steps (reference
    test_paper_stack_vda_ops.py:300-323)."""
    from vdn_b200.linear_attention import vda_gather, vda_scan, window_bounds
    from vdn_b200.paper_factor import paper_delta_factors
    torch.manual_seed(102)
    frames, h, d = 102, 1, 128
    k = torch.randn(frames, h, 7, d) * .025
    a = (k.transpose(-1, -2) @ k).contiguous()
    b = torch.randn_like(a) * .01
    alpha = torch.rand(frames, h, d) * .01 + .99
    t, inj = paper_delta_factors(a.to(cuda), b.to(cuda), alpha.to(cuda))
    seed = torch.randn(h, d, d)
    prefix, suffix = vda_scan(t, inj, seed.to(cuda))
    op, osf = ovda.run_scans(t.double().cpu().numpy(), inj.double().cpu().numpy(), seed.double().numpy())
    torch.testing.assert_close(prefix.double().cpu(), torch.from_numpy(op), atol=4e-6, rtol=1e-4)
    torch.testing.assert_close(suffix.double().cpu(), torch.from_numpy(osf), atol=4e-6, rtol=1e-4)
    bounds = window_bounds(frames, 1, 5)
    got = vda_gather(prefix, suffix, alpha.to(cuda), bounds, seed.to(cuda), torch.float32)
    want = ovda.gather(op, osf, alpha.numpy(), bounds, seed.double().numpy())
    assert rel_l2(got.cpu().numpy(), want) < 5e-6


@torch.no_grad()
def test_head_shard_and_nondefault_stream(cuda, vda_golden):
    """Head slices of a strided packed buffer on a side stream equal the full call."""
    from vdn_b200.linear_attention import BidirectionalLinearBranch
    c = _case(vda_golden, "d128_wide", cuda)
    branch = BidirectionalLinearBranch(16, c["h"], c["d"]).to(cuda)
    alpha = c["alpha"]
    branch.alpha.forward = lambda fm, heads=None: alpha if heads is None else alpha[:, heads]
    mean = torch.zeros(c["f"], 16, device=cuda)
    full = branch(None, c["f"], c["s"], c["bounds"], (c["q"], c["k"], c["v"]),
                  heads=slice(0, c["h"]), beta=c["beta"], gate=c["gate"], frame_mean=mean)
    packed = torch.cat([c["q"], c["k"], c["v"]], dim=-1)      # [T, H, 3d] strided fields
    q, k, v = packed.split(c["d"], dim=-1)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        part = branch(None, c["f"], c["s"], c["bounds"], (q[:, 1:2], k[:, 1:2], v[:, 1:2]),
                      heads=slice(1, 2), beta=c["beta"][:, 1:2], gate=c["gate"][:, 1:2],
                      frame_mean=mean)
    torch.cuda.current_stream().wait_stream(stream)
    want = full.view(-1, c["h"], c["d"])[:, 1].reshape_as(part)
    assert rel_l2(part.float().cpu().numpy(), want.float().cpu().numpy()) < 1e-6


@torch.no_grad()
def test_full_size_config2_properties(cuda):
    """BASELINE config 2 (H=40, d=128, 21 x 1560 tokens): finite output, exact
    head independence (a 2-head slice equals the full call's slice), and parity
    of one frame-window against the oracle on a reduced sub-problem."""
    from vdn_b200.linear_attention import vda_forward, window_bounds
    f, s, h, d = 21, 1560, 40, 128
    g = torch.Generator(device=cuda).manual_seed(2)
    n = f * s
    q = F.normalize(torch.randn(n, h, d, device=cuda, generator=g), dim=-1).bfloat16()
    k = F.normalize(torch.randn(n, h, d, device=cuda, generator=g), dim=-1).bfloat16()
    v = torch.randn(n, h, d, device=cuda, generator=g).bfloat16()
    beta = torch.sigmoid(torch.randn(n, h, device=cuda, generator=g)).bfloat16()
    gate = torch.rand(n, h, d, device=cuda, generator=g).bfloat16()
    alpha = torch.exp(-F.softplus(torch.randn(f, h, 1, device=cuda, generator=g))).expand(f, h, d)
    w = torch.ones(d, device=cuda)
    bounds = window_bounds(f, 1)
    out = vda_forward(q, k, v, beta, gate, alpha, bounds, f, s, w)
    assert out.shape == (n, h * d) and bool(torch.isfinite(out).all())
    sl = slice(7, 9)
    part = vda_forward(q[:, sl], k[:, sl], v[:, sl], beta[:, sl], gate[:, sl], alpha[:, sl],
                       bounds, f, s, w)
    assert torch.equal(part, out.view(n, h, d)[:, sl].reshape(n, -1))
    ref = ovda.readout(q[:, 7:8].float().cpu().numpy(), k[:, 7:8].float().cpu().numpy(),
                       v[:, 7:8].float().cpu().numpy(), beta[:, 7:8].float().cpu().numpy(),
                       gate[:, 7:8].float().cpu().numpy(), alpha[:, 7:8].float().cpu().numpy(),
                       bounds, f, s)
    got = out.view(n, h, d)[:, 7].float().cpu().numpy()
    assert rel_l2(got, ref.reshape(n, d)) < 4e-3


# ------------------------------------------------------- tensor-core factor + scan
@pytest.mark.parametrize("frames,heads,tokens,beta_scale", [(3, 2, 40, 1.0), (5, 3, 1008, 50.0)])
def test_factor_inverse_planes_equal_factor_kernel(cuda, frames, heads, tokens, beta_scale):
    """The split planes of vdn_vda_factor_inverse sum exactly to the fp32 inverse the
    T / J factor kernel computes (the same Gauss-Jordan arithmetic), and that inverse
    matches fp64."""
    from vdn_b200.linear_attention import split_inverse_values, vda_factor_inverse
    from vdn_b200.paper_factor import paper_delta_factors
    A, B, _ = _stats_inputs(frames, heads, tokens, beta_scale, d=128)
    planes = vda_factor_inverse(A.to(cuda))
    inv = split_inverse_values(planes)
    t, _ = paper_delta_factors(A.to(cuda), B.to(cuda), None)
    assert torch.equal(inv, t)
    ref, _ = _fp64_factors(A, B)
    assert rel_l2(inv.double().cpu().numpy(), ref.numpy()) < 1e-5


@pytest.mark.parametrize("frames", [1, 2, 11, 31])
@pytest.mark.parametrize("text", [False, True])
@pytest.mark.parametrize("decay", [1.0, 0.7, 0.001])
def test_scan_tc_vs_fp64(cuda, frames, text, decay):
    """The tensor-core scan (three-way bf16 split products, fp32 accumulation) against
    the fp64 recurrence on the same inverse: T = diag(alpha) inv^T, J = B inv^T (the MMA
    reads the inverse's rows as the B operand), the reference's scan limits."""
    from vdn_b200.linear_attention import split_inverse_values, vda_factor_inverse, vda_scan_tc
    torch.manual_seed(frames)
    h, d = 2, 128
    k = F.normalize(torch.randn(frames, h, 9, d), dim=-1)
    a = (k.transpose(-1, -2) @ k).contiguous()
    b = torch.randn_like(a) * 0.1
    alpha = (torch.rand(frames, h, d) * 0.1 + 0.9) * decay
    planes = vda_factor_inverse(a.to(cuda))
    inv = split_inverse_values(planes).double().cpu()
    t = alpha.double()[..., :, None] * inv.transpose(-1, -2)
    j = b.double() @ inv.transpose(-1, -2)
    seed = torch.randn(h, d, d) * .3 if text else None
    prefix, suffix = vda_scan_tc(planes, b.to(cuda), alpha.to(cuda), None if seed is None else seed.to(cuda))
    op, osf = ovda.run_scans(t.numpy(), j.numpy(), None if seed is None else seed.double().numpy())
    torch.testing.assert_close(prefix.double().cpu(), torch.from_numpy(op), atol=3e-6, rtol=3e-5)
    torch.testing.assert_close(suffix.double().cpu(), torch.from_numpy(osf), atol=3e-6, rtol=3e-5)


@pytest.mark.parametrize("frames,heads,text", [(21, 4, False), (3, 1, True), (70, 2, False)])
def test_scan_tc_bf16_b_equals_fp32_b(cuda, frames, heads, text):
    """B in bf16 (staged by TMA, the forward's form) gives exactly the banks of the fp32-B
    path fed the same bf16 values (the statistics produce bf16-valued B either way)."""
    from vdn_b200.linear_attention import vda_factor_inverse, vda_scan_tc
    g = torch.Generator().manual_seed(frames * 7 + heads)
    k = F.normalize(torch.randn(frames, heads, 16, 128, generator=g), dim=-1)
    a = (k.transpose(-1, -2) @ k).contiguous()
    b = (torch.randn(a.shape, generator=g) * 0.1).bfloat16()
    alpha = torch.rand(frames, heads, 128, generator=g) * 0.2 + 0.8
    seed = torch.randn(heads, 128, 128, generator=g) * .3 if text else None
    planes = vda_factor_inverse(a.to(cuda))
    s = None if seed is None else seed.to(cuda)
    p32, s32 = vda_scan_tc(planes, b.float().to(cuda), alpha.to(cuda), s)
    p16, s16 = vda_scan_tc(planes, b.to(cuda), alpha.to(cuda), s)
    torch.cuda.synchronize()
    assert torch.equal(p16, p32) and torch.equal(s16, s32)


@pytest.mark.parametrize("heads", [1, 5, 40, 80])
def test_scan_tc_head_counts_and_long_recurrence(cuda, heads):
    """Every head count (one CTA per head and direction: 2 to 160 CTAs) and a long
    recurrence near identity (102 frames at one head, reference test_paper_stack_vda_ops.py:300-323)."""
    from vdn_b200.linear_attention import split_inverse_values, vda_factor_inverse, vda_scan_tc
    frames = 102 if heads == 1 else 5
    g = torch.Generator().manual_seed(heads)
    k = torch.randn(frames, heads, 7, 128, generator=g) * (.025 if heads == 1 else .3)
    a = (k.transpose(-1, -2) @ k).contiguous()
    b = torch.randn(a.shape, generator=g) * (.01 if heads == 1 else .1)
    alpha = torch.rand(frames, heads, 128, generator=g) * .01 + .99
    seed = torch.randn(heads, 128, 128, generator=g) * .3
    planes = vda_factor_inverse(a.to(cuda))
    inv = split_inverse_values(planes).double().cpu()
    t = alpha.double()[..., :, None] * inv.transpose(-1, -2)
    j = b.double() @ inv.transpose(-1, -2)
    prefix, suffix = vda_scan_tc(planes, b.to(cuda), alpha.to(cuda), seed.to(cuda))
    op, osf = ovda.run_scans(t.numpy(), j.numpy(), seed.double().numpy())
    tol = dict(atol=4e-6, rtol=1e-4) if heads == 1 else dict(atol=3e-6, rtol=3e-5)
    torch.testing.assert_close(prefix.double().cpu(), torch.from_numpy(op), **tol)
    torch.testing.assert_close(suffix.double().cpu(), torch.from_numpy(osf), **tol)
