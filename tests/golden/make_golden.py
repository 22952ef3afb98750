"""Generate the golden fixtures under tests/golden/ from the REFERENCE's own CPU code.

Run once, in a container where the reference checkout is importable:

    python tests/golden/make_golden.py /path/to/vdn/checkout

It imports the reference (ec-jt/vdn) and records, on seeded synthetic inputs:
  * quantize_cpu codes/scales (src/models/ops/mxfp8_quant.py:40-74) for the
    BASELINE config-0 256x256 matrix, odd shapes, an outlier matrix and the
    exponent-boundary known-answer vector;
  * the eager VDA body BidirectionalLinearBranch._readout
    (src/models/linear_attention/branch.py:404-482) with alpha injected, at the
    BASELINE config-0 geometry (F=4, S=64, H=4, d=64) and at d=128 with and
    without the text seed and the anchor frames;
  * the stage functions frame_statistics, VdnDelta.factor_apply, _run_scans and
    gather_linear_state (scan.py, delta_rule.py) on one d=128 case;
  * the separable short conv LinearAttentionSepConv (features.py:133-209): its
    spatial 5x5 half, the eager temporal 5-tap shift and the activated k / v
    features, on two grids (--sepconv-only regenerates just these);
  * window_softmax_reference (src/models/softmax_attention/window.py:56-111) with
    global text rows, frame and chunk-aligned windows and every anchor mode
    (--window-only regenerates just these);
  * FrameKDAAlpha.forward (src/models/linear_attention/layers.py:36-69): its seeded
    weights, frame means and alpha, for all heads and for a head range
    (--alpha-only regenerates just these).

Nothing at test time reads the reference; the tests read only these .npz files.
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 tensor -> uint16 bit patterns."""
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def mxfp8_fixtures(quantize_cpu):
    out = {}
    g = torch.Generator().manual_seed(0)
    x = torch.randn(256, 256, generator=g).bfloat16()
    q, s = quantize_cpu(x)
    out.update(cfg0_x=bits(x), cfg0_q=q.numpy(), cfg0_s=s.numpy())
    for i, shape in enumerate([(1, 1), (3, 31), (127, 32), (129, 129), (9, 256), (130, 300)]):
        x = torch.randn(shape, generator=g).bfloat16()
        q, s = quantize_cpu(x, chunk_rows=7)
        out[f"shape{i}_x"], out[f"shape{i}_q"], out[f"shape{i}_s"] = bits(x), q.numpy(), s.numpy()
    # BASELINE config-1 activation distribution: N(0,1) with 1% of channels x50.
    x = torch.randn(200, 640, generator=g)
    idx = torch.randperm(640, generator=g)[:640 // 100]
    x[:, idx] *= 50
    x = x.bfloat16()
    q, s = quantize_cpu(x)
    out.update(outlier_x=bits(x), outlier_q=q.numpy(), outlier_s=s.numpy())
    # Exponent boundaries (reference test_paper_stack_mxfp8_ops.py:67-78), plus
    # subnormal, negative-zero and mixed-sign rows.
    kat = torch.tensor([0., 224., 448., 449., 896., 1e-38, -3.0e-39, -0.0, 1.75, -1.7501],
                       dtype=torch.float32)[:, None].expand(-1, 32).contiguous()
    kat[8, ::2] *= -1
    q, s = quantize_cpu(kat)
    out.update(kat_x=kat.numpy(), kat_q=q.numpy(), kat_s=s.numpy())
    np.savez_compressed(HERE / "mxfp8_golden.npz", **out)


def vda_case(branch_cls, f, s, h, d, seed, text_len=0, skip_ends=False, radius=1):
    g = torch.Generator().manual_seed(seed)
    n = f * s

    def raw_qk():
        # BASELINE: q,k ~ N(0,1) bf16, L2-normalised per head, then given to the op.
        return F.normalize(torch.randn(n, h, d, generator=g), dim=-1).bfloat16()

    q, k = raw_qk(), raw_qk()
    v = torch.randn(n, h, d, generator=g).bfloat16()
    beta = torch.sigmoid(torch.randn(n, h, generator=g)).bfloat16()
    gate = torch.rand(n, h, d, generator=g).bfloat16()
    # log alpha = -softplus(N(0,1)) per (frame, head), broadcast over d_k.
    alpha = torch.exp(-F.softplus(torch.randn(f, h, 1, generator=g))).expand(f, h, d).contiguous()
    bounds = [(t - radius, t + radius) for t in range(f)]
    text = {}
    if text_len:
        tq, tk = (F.normalize(torch.randn(text_len, h, d, generator=g), dim=-1).bfloat16()
                  for _ in range(2))
        tv = torch.randn(text_len, h, d, generator=g).bfloat16()
        tb = torch.sigmoid(torch.randn(text_len, h, generator=g)).bfloat16()
        text = dict(text_qkv_raw=(tq, tk, tv), text_beta=tb)
    hidden = 16
    branch = branch_cls(hidden, h, d, delta_rule="vdn_solve").eval()
    branch.alpha.forward = lambda frame_mean, heads=None: alpha[1:-1] if (
        skip_ends and frame_mean.shape[0] == f - 2) else alpha
    with torch.no_grad():
        out = branch(None, f, s, bounds, (q, k, v), skip_ends=skip_ends,
                     heads=slice(0, h), beta=beta, gate=gate,
                     frame_mean=torch.zeros(f, hidden), **text)
    rec = dict(q=bits(q), k=bits(k), v=bits(v), beta=bits(beta), gate=bits(gate),
               alpha=alpha.numpy(), bounds=np.array(bounds, np.int64),
               geometry=np.array([f, s, h, d, int(skip_ends), text_len], np.int64),
               out=bits(out))
    if text_len:
        rec.update(tk=bits(text["text_qkv_raw"][1]), tv=bits(text["text_qkv_raw"][2]),
                   tbeta=bits(text["text_beta"]))
    return rec


def stage_fixtures(scan, delta):
    g = torch.Generator().manual_seed(5)
    f, h, s, d = 5, 1, 40, 128
    k = F.normalize(F.silu(torch.randn(f, h, s, d, generator=g)), dim=-1).bfloat16()
    v = F.silu(torch.randn(f, h, s, d, generator=g)).bfloat16()
    beta = torch.sigmoid(torch.randn(f, h, s, generator=g)).bfloat16()
    alpha = (torch.rand(f, h, d, generator=g) * 0.5 + 0.45).float()
    with torch.no_grad():
        a, b = scan.frame_statistics(k, v, beta, a_fp32=True)
        t, j = delta.VdnDelta().factor_apply(alpha, a, b)
        seed = torch.randn(h, d, d, generator=g) * 0.1
        prefix, suffix = scan._run_scans(delta.VdnDelta(), alpha, a, b, text_state=seed)
        bounds = [(t_ - 1, t_ + 2) for t_ in range(f)]
        gathered = scan.gather_linear_state(prefix, suffix, alpha, bounds, text_state=seed)
        gathered0 = scan.gather_linear_state(prefix, suffix, alpha, bounds, text_state=None)
    np.savez_compressed(
        HERE / "vda_stages_golden.npz", k=bits(k), v=bits(v), beta=bits(beta),
        alpha=alpha.numpy(), a=a.numpy(), b=b.numpy(), t=t.numpy(), j=j.numpy(),
        seed=seed.numpy(), prefix=prefix.numpy(), suffix=suffix.numpy(),
        bounds=np.array(bounds, np.int64), gathered=gathered.numpy(),
        gathered_noseed=gathered0.numpy())


def sepconv_fixtures(features_mod):
    """Reference short conv on CPU: spatial half (bf16 conv2d), eager temporal shift,
    and prepare_linear_features (conv -> SiLU [-> L2Norm]) for k and v."""
    out = {}
    cases = {"small": dict(f=4, gh=6, gw=8, h=2, d=64, seed=21),
             "d128": dict(f=5, gh=5, gw=7, h=2, d=128, seed=22)}
    for name, c in cases.items():
        torch.manual_seed(c["seed"])
        ch = c["h"] * c["d"]
        conv = features_mod.LinearAttentionSepConv(ch, ("k", "v")).to(torch.bfloat16)
        s = c["gh"] * c["gw"]
        g = torch.Generator().manual_seed(c["seed"] + 100)
        for proj in ("k", "v"):
            tokens = torch.randn(c["f"] * s, c["h"], c["d"], generator=g).bfloat16()
            with torch.no_grad():
                x, w_tm = conv.spatial(proj, tokens, c["f"], (c["gh"], c["gw"]))
                tm = features_mod._temporal_shift(x, w_tm, 5, 2)
                feat = features_mod.prepare_linear_features(
                    tokens, l2norm=(proj != "v"), conv=conv, proj=proj, num_frames=c["f"],
                    frame_size=(c["gh"], c["gw"]))
            key = f"{name}_{proj}"
            out[f"{key}_x"] = bits(tokens)
            out[f"{key}_wsp"] = bits(getattr(conv, f"{proj}_sp").weight.detach())
            out[f"{key}_wtm"] = bits(getattr(conv, f"{proj}_tm").weight.detach())
            out[f"{key}_spatial"] = bits(x)
            out[f"{key}_temporal"] = bits(tm)
            out[f"{key}_features"] = bits(feat)
        out[f"{name}_geom"] = np.array([c["f"], c["gh"], c["gw"], c["h"], c["d"]], dtype=np.int64)
    np.savez_compressed(HERE / "sepconv_golden.npz", **out)


WINDOW_CASES = {
    # name: text rows, frames, tokens per frame, heads, head dim, radius, chunk, anchors
    "frame_text_both": (5, 6, 8, 2, 16, 1, 0, "both"),
    "chunk_text_columns": (3, 7, 6, 2, 16, 1, 2, "columns"),
    "frame_rows": (0, 5, 8, 3, 16, 0, 0, "rows"),
    "frame_text_none": (4, 4, 8, 2, 16, 1, 0, "none"),
    "chunk_both_short_last": (2, 5, 4, 2, 32, 0, 2, "both"),
}


def window_fixtures(ref_root: str):
    """window_softmax_reference (src/models/softmax_attention/window.py:56-111) on CPU,
    fp32, with global text rows first, frame and chunk-aligned windows and every
    anchor mode.  The module is loaded from its file: the package __init__ imports
    diffusers."""
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "ref_window", str(Path(ref_root) / "src/models/softmax_attention/window.py"))
    win = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(win)
    from src.models.sequence_layout import SequenceLayout
    out = {}
    for i, (name, (L, f, s, h, d, radius, chunk, anchors)) in enumerate(WINDOW_CASES.items()):
        g = torch.Generator().manual_seed(300 + i)
        n = L + f * s
        q, k, v = (torch.randn(n, h, d, generator=g) for _ in range(3))
        layout = SequenceLayout(seq_len=n, video_start=L, num_frames=f, tokens_per_frame=s,
                                text_start=0, text_len=L)
        bounds = win.window_bounds(f, radius, chunk)
        with torch.no_grad():
            o = win.window_softmax_reference(q, k, v, layout, bounds, d ** -0.5, anchor_frames=anchors)
        out[f"{name}_q"], out[f"{name}_k"], out[f"{name}_v"] = q.numpy(), k.numpy(), v.numpy()
        out[f"{name}_out"] = o.numpy()
        out[f"{name}_geom"] = np.array([L, f, s, h, d, radius, chunk], np.int64)
        out[f"{name}_bounds"] = np.array(bounds, np.int64)
        out[f"{name}_anchors"] = np.array(anchors)
    np.savez_compressed(HERE / "window_golden.npz", **out)


def alpha_fixtures(layers_mod):
    """FrameKDAAlpha at its own init (torch default Linear init, fla A_log / dt_bias),
    on frame means of two magnitudes (block-like means and large ones that reach the
    softplus tail), for every head and for the head range [1, 3)."""
    out = {}
    cases = {"small": dict(hidden=256, heads=4, d=64, frames=5, scale=0.05, seed=31),
             "d128": dict(hidden=512, heads=4, d=128, frames=7, scale=3.0, seed=32)}
    for name, c in cases.items():
        torch.manual_seed(c["seed"])
        mod = layers_mod.FrameKDAAlpha(c["hidden"], c["heads"], c["d"])
        g = torch.Generator().manual_seed(c["seed"] + 100)
        fm = torch.randn(c["frames"], c["hidden"], generator=g) * c["scale"]
        with torch.no_grad():
            full = mod(fm)
            part = mod(fm, heads=slice(1, 3))
        out.update({f"{name}_down": mod.down.weight.detach().numpy(),
                    f"{name}_up": mod.up.weight.detach().numpy(),
                    f"{name}_a_log": mod.A_log.detach().numpy(),
                    f"{name}_dt_bias": mod.dt_bias.detach().numpy(),
                    f"{name}_frame_mean": fm.numpy(), f"{name}_alpha": full.numpy(),
                    f"{name}_alpha_heads13": part.numpy(),
                    f"{name}_geometry": np.array([c["hidden"], c["heads"], c["d"]])})
    np.savez_compressed(HERE / "alpha_golden.npz", **out)


def main(ref_root: str, sepconv_only: bool = False, window_only: bool = False,
         alpha_only: bool = False):
    sys.path.insert(0, ref_root)
    torch.set_num_threads(8)
    from src.models.linear_attention import layers as layers_mod
    alpha_fixtures(layers_mod)
    if alpha_only:
        print("wrote alpha_golden.npz")
        return
    if window_only:
        window_fixtures(ref_root)
        print("wrote window_golden.npz")
        return
    from src.models.linear_attention import features as features_mod
    sepconv_fixtures(features_mod)
    if sepconv_only:
        print("wrote sepconv_golden.npz")
        return
    window_fixtures(ref_root)
    from src.models.ops.mxfp8_quant import quantize_cpu
    from src.models.linear_attention import scan, delta_rule
    from src.models.linear_attention.branch import BidirectionalLinearBranch

    torch.set_num_threads(8)
    mxfp8_fixtures(quantize_cpu)
    cases = {
        "cfg0": dict(f=4, s=64, h=4, d=64, seed=10),
        "d128": dict(f=5, s=40, h=2, d=128, seed=11),
        "d128_text": dict(f=5, s=24, h=2, d=128, seed=12, text_len=7),
        "d128_anchor": dict(f=6, s=16, h=2, d=128, seed=13, skip_ends=True),
        "d128_wide": dict(f=7, s=20, h=3, d=128, seed=14, radius=2),
    }
    recs = {}
    for name, kw in cases.items():
        for key, val in vda_case(BidirectionalLinearBranch, **kw).items():
            recs[f"{name}_{key}"] = val
    np.savez_compressed(HERE / "vda_golden.npz", **recs)
    stage_fixtures(scan, delta_rule)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    if len(args) != 1:
        raise SystemExit("usage: make_golden.py <path to the ec-jt/vdn checkout> "
                         "[--sepconv-only | --window-only | --alpha-only]")
    main(args[0], sepconv_only="--sepconv-only" in sys.argv, window_only="--window-only" in sys.argv,
         alpha_only="--alpha-only" in sys.argv)
