"""CPU: the oracle against the reference's golden fixtures and known-answer tests.

The fixtures were produced by the reference's own code (tests/golden/make_golden.py);
the KATs restate tests/test_paper_stack_mxfp8_ops.py:67-83 of the reference.
"""
import numpy as np
import pytest

from oracle import mxfp8 as mx
from oracle import vda
from helpers import rel_l2, max_abs

MX_CASES = ["cfg0", "outlier", "kat"] + [f"shape{i}" for i in range(6)]
VDA_CASES = ["cfg0", "d128", "d128_text", "d128_anchor", "d128_wide"]


def _x(g, name):
    a = g[name]
    return mx.bf16_to_f32(a) if a.dtype == np.uint16 else a


@pytest.mark.parametrize("case", MX_CASES)
def test_quantiser_oracle_bit_exact_vs_reference(mxfp8_golden, case):
    q, s = mx.quantize(_x(mxfp8_golden, case + "_x"))
    assert np.array_equal(q, mxfp8_golden[case + "_q"])
    assert np.array_equal(s, mxfp8_golden[case + "_s"])


def test_exponent_boundaries_kat():
    # reference tests/test_paper_stack_mxfp8_ops.py:67-78
    values = np.array([0., 224., 448., 449., 896., 1e-38], np.float32)
    x = np.repeat(values[:, None], 32, 1)
    q, s = mx.quantize(x)
    natural = mx.unswizzle(s, *q.shape)
    assert natural[:5, 0].tolist() == [0, 126, 127, 128, 128]
    assert np.isfinite(mx.dequantize(q, s)).all()
    for i in range(5):
        e = int(natural[i, 0]) - 127
        assert np.array_equal(q[i, :32], mx.f32_to_e4m3_bits(x[i] * np.float32(2.0 ** -e)))


def test_swizzle_unique_address_oracle():
    natural = (np.arange(256 * 12) % 251).astype(np.uint8).reshape(256, 12)
    assert np.array_equal(mx.unswizzle(mx.swizzle(natural), 256, 384), natural)


def test_padding_and_dequant_roundtrip():
    rng = np.random.default_rng(13)
    for shape in [(1, 1), (3, 31), (127, 32), (129, 129), (9, 256)]:
        x = mx.round_bf16(rng.standard_normal(shape).astype(np.float32))
        q, s = mx.quantize(x)
        back = mx.dequantize(q, s)
        assert np.count_nonzero(back[shape[0]:]) == 0 and np.count_nonzero(back[:, shape[1]:]) == 0
        np.testing.assert_allclose(back[:shape[0], :shape[1]], x, rtol=.063, atol=.001)


@pytest.mark.parametrize("value", [np.nan, np.inf, -np.inf])
def test_reject_nonfinite(value):
    with pytest.raises(ValueError, match="nonfinite"):
        mx.quantize(np.array([[value]], np.float32))


def test_e4m3_conversion_exhaustive_against_decode():
    # Every finite E4M3 code decodes and re-encodes to itself; midpoints round to even.
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], np.uint8)
    vals = mx.e4m3_bits_to_f32(codes)
    assert np.array_equal(mx.f32_to_e4m3_bits(vals), codes)
    pos = np.sort(mx.e4m3_bits_to_f32(np.arange(0, 0x7F, dtype=np.uint8)))
    mids = ((pos[:-1].astype(np.float64) + pos[1:]) / 2).astype(np.float32)
    got = mx.e4m3_bits_to_f32(mx.f32_to_e4m3_bits(mids))
    lower_even = (mx.f32_to_e4m3_bits(pos[:-1]) & 1) == 0
    np.testing.assert_array_equal(got, np.where(lower_even, pos[:-1], pos[1:]))


def _vda_inputs(g, name):
    f, s, h, d, skip, tl = (int(x) for x in g[name + "_geometry"])
    b = lambda k: mx.bf16_to_f32(g[name + "_" + k])
    seed = None
    if tl:
        seed = vda.text_seed(b("tk").reshape(tl, h, d), b("tv").reshape(tl, h, d), b("tbeta"))
    return dict(q_raw=b("q"), k_raw=b("k"), v_raw=b("v"), beta=b("beta"), gate=b("gate"),
                alpha=g[name + "_alpha"], bounds=[tuple(x) for x in g[name + "_bounds"]],
                num_frames=f, tokens_per_frame=s, skip_ends=bool(skip), seed=seed), b("out")


@pytest.mark.parametrize("case", VDA_CASES)
def test_vda_oracle_vs_reference_branch(vda_golden, case):
    kw, ref = _vda_inputs(vda_golden, case)
    out = vda.branch_forward(**kw)
    # bf16 rounding points flip by one ulp between fp64 and the reference's fp32.
    assert rel_l2(out, ref) < 1e-3
    assert max_abs(out, ref) <= 0.03125


def test_vda_oracle_stages_vs_reference(vda_stages_golden):
    g = vda_stages_golden
    k, v, beta = (mx.bf16_to_f32(g[n]) for n in ("k", "v", "beta"))
    a, b = vda.frame_statistics(k, v, beta)
    assert rel_l2(a, g["a"]) < 1e-6 and rel_l2(b, g["b"]) < 1e-6
    t, j = vda.delta_factors(g["a"], g["b"], g["alpha"])
    assert rel_l2(t, g["t"]) < 1e-5 and rel_l2(j, g["j"]) < 3e-5
    p, sf = vda.run_scans(g["t"].astype(np.float64), g["j"].astype(np.float64), g["seed"])
    assert rel_l2(p, g["prefix"]) < 1e-6 and rel_l2(sf, g["suffix"]) < 1e-6
    bounds = [tuple(x) for x in g["bounds"]]
    pre, suf = g["prefix"].astype(np.float64), g["suffix"].astype(np.float64)
    assert rel_l2(vda.gather(pre, suf, g["alpha"], bounds, g["seed"]), g["gathered"]) < 1e-6
    assert rel_l2(vda.gather(pre, suf, g["alpha"], bounds, None), g["gathered_noseed"]) < 1e-6


def test_window_bounds_chunk_mode():
    # reference window.py:26-52 and test_paper_stack_vda_ops.py:290-296
    assert vda.window_bounds(4, 1) == [(-1, 1), (0, 2), (1, 3), (2, 4)]
    b = vda.window_bounds(12, 1, 5)
    assert b[5] == b[9] == (0, 14) and b[10] == (5, 19)


@pytest.mark.parametrize("case", ["small", "d128"])
def test_frame_alpha_oracle_vs_reference(alpha_golden, case):
    """oracle.vda.frame_alpha against FrameKDAAlpha.forward run by the reference
    (layers.py:36-69), for every head and for the head range [1, 3)."""
    g = alpha_golden
    hidden, heads, d = (int(x) for x in g[case + "_geometry"])
    up, dt = g[case + "_up"], g[case + "_dt_bias"]
    got = vda.frame_alpha(g[case + "_frame_mean"], g[case + "_down"], up, dt, g[case + "_a_log"], heads, d)
    want = g[case + "_alpha"]
    assert got.shape == want.shape
    np.testing.assert_allclose(got, want, rtol=2e-6, atol=1e-7)
    rows = slice(1 * d, 3 * d)
    part = vda.frame_alpha(g[case + "_frame_mean"], g[case + "_down"], up[rows], dt[rows],
                           g[case + "_a_log"][1:3], 2, d)
    np.testing.assert_allclose(part, g[case + "_alpha_heads13"], rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("case", MX_CASES)
def test_qdq_torch_matches_numpy_oracle(mxfp8_golden, case):
    """The torch CPU restatement used by the full-size checks gives exactly the values of
    dequantize(quantize(x)) on every fixture."""
    import torch
    x = _x(mxfp8_golden, case + "_x")
    r, k = x.shape
    want = mx.dequantize(*mx.quantize(x))[:r, :k].astype(np.float32)
    got = mx.qdq_torch(torch.from_numpy(np.ascontiguousarray(x, np.float32))).numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_qdq_torch_random_and_subnormal_blocks():
    import torch
    g = torch.Generator().manual_seed(7)
    x = torch.randn(300, 640, generator=g) * torch.exp2(torch.randint(-140, 100, (300, 1), generator=g).float())
    x[5, :32] = 0.0
    x[6, :32] = -0.0
    x = x.bfloat16().float()
    want = mx.dequantize(*mx.quantize(x.numpy()))[:300, :640].astype(np.float32)
    got = mx.qdq_torch(x).numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


@pytest.mark.parametrize("text_rows,chunk", [(0, 0), (24, 0), (0, 2)])
def test_block_oracle_sampled_frames_equal_full(text_rows, chunk):
    """block_reference(out_frames=...) returns exactly the full evaluation's rows of those
    frames (the full-size GPU checks rely on it)."""
    import types
    import torch
    from oracle import block as oblock
    cfg = types.SimpleNamespace(hidden=256, heads=2, head_dim=128, ffn=512, radius=1, eps=1e-6,
                                gelu="tanh", chunk=chunk, anchor_frames="none", text_state=bool(text_rows))
    g = torch.Generator().manual_seed(3)
    hd, H, d, ffn = 256, 2, 128, 512
    r = lambda *s, std=0.05: torch.randn(*s, generator=g) * std
    w = dict(adaln_w=r(6 * hd, hd), adaln_b=r(6 * hd), norm1=torch.ones(hd), norm2=torch.ones(hd),
             qkv=r(3 * hd, hd), qkv_b=r(3 * hd), o=r(hd, hd), ol=r(hd, hd), o_b=r(hd), o_b_softmax=r(hd),
             up=r(ffn, hd), up_b=r(ffn), down=r(hd, ffn), down_b=r(hd), sg_w=r(H, hd), sg_b=r(H),
             beta_w=r(H, hd), og_down=r(d, hd), og_up=r(hd, d), og_b=r(hd))
    frames, tokens = 5, 16
    x = torch.randn(text_rows + frames * tokens, hd, generator=g).bfloat16()
    temb = torch.randn(hd, generator=g)
    alpha = lambda fm: torch.full((frames, H, d), 0.9)
    full = oblock.block_reference(x, temb, w, frames, tokens, cfg, alpha, text_rows=text_rows)
    pick = [4, 0, 2]
    part = oblock.block_reference(x, temb, w, frames, tokens, cfg, alpha, text_rows=text_rows,
                                  out_frames=pick)
    want = torch.cat([full[text_rows + f * tokens:text_rows + (f + 1) * tokens] for f in pick])
    assert torch.equal(part, want)


@pytest.mark.parametrize("case", ["d128", "d128_wide", "d128_text"])
def test_vda_oracle_out_frames_equal_full(vda_golden, case):
    """readout(out_frames=...) gives exactly the full readout's rows of those frames."""
    kw, _ = _vda_inputs(vda_golden, case)
    full = vda.branch_forward(**kw)
    f, s = kw["num_frames"], kw["tokens_per_frame"]
    part = vda.branch_forward(**kw, out_frames=[f - 1, 0])
    for fr in (f - 1, 0):
        assert np.array_equal(part[fr * s:(fr + 1) * s], full[fr * s:(fr + 1) * s])


def test_round_bf16_matches_bit_formula():
    g = np.random.default_rng(5)
    x = (g.standard_normal(200_000) * np.exp2(g.integers(-130, 120, 200_000))).astype(np.float32)
    x[:4] = [0.0, -0.0, 1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8]   # ties round to even
    assert np.array_equal(mx.round_bf16(x).view(np.uint32), mx.bf16_to_f32(mx.f32_to_bf16_bits(x)).view(np.uint32))
