"""CPU fp32 reference of the hybrid DiT block. TEST INFRASTRUCTURE ONLY.

Composition of the reference pieces (ec-jt/vdn), evaluated in fp32 on the CPU
with the MXFP8 quantisation points of the B200 path reproduced bit-exactly by
oracle.mxfp8 (so the GEMM inputs match) and the VDA branch by oracle.vda:

  AdaLN modulation ........ bf16 SiLU of the timestep embedding, then the bf16 projection
                            (block.adaln_proj(temb), src/models/ops/fused_block.py:118)
  pre-norm + AdaLN ........ src/models/ops/fused_block.py:43-46 (_pre_ref)
  MXFP8 linears ........... src/models/ops/mxfp8_linear.py:60-102 (dequantised GEMM)
  window softmax .......... src/models/softmax_attention/window.py:56-111
  softmax gate ............ src/models/attention_gates.py:13-55, hybrid_attention.py:217-222
  linear branch ........... src/models/linear_attention/branch.py (oracle.vda)
  output merge ............ src/models/hybrid_attention.py:250-255 (to_out + to_out_linear)
  gated residual .......... src/models/ops/fused_block.py:49-51 (_post_ref)
  GELU FFN ................ the BASELINE block's FFN (tanh GELU)
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import mxfp8 as omx
from . import vda as ovda


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).float()


def _qdq(x: torch.Tensor) -> torch.Tensor:
    """Activation through the MXFP8 quantiser and back (fp32 values of the codes);
    oracle.mxfp8.qdq_torch, bit-exact with dequantize(quantize(x))."""
    return omx.qdq_torch(x.float())


def _linear(x_dq, w_dq, bias):
    y = _bf16(x_dq @ w_dq.T)
    return y if bias is None else _bf16(y + bias.float())


def prenorm(x, weight, scale, shift, eps):
    x = x.float()
    inv = torch.rsqrt(x.square().mean(-1, keepdim=True) + eps)
    return _bf16((x * inv * weight.float()) * (1 + scale.float()) + shift.float())


def window_attention(q, k, v, frames, tokens, radius, scale, only_frames=None):
    """Exact windowed softmax, one SDPA per query frame, fp32. q/k/v [T, H, d].
    only_frames: compute those query frames only (other rows are left zero)."""
    out = torch.zeros_like(q)
    for f in (range(frames) if only_frames is None else only_frames):
        lo, hi = max(0, f - radius), min(frames - 1, f + radius)
        qs = q[f * tokens:(f + 1) * tokens].permute(1, 0, 2)
        ks = k[lo * tokens:(hi + 1) * tokens].permute(1, 0, 2)
        vs = v[lo * tokens:(hi + 1) * tokens].permute(1, 0, 2)
        out[f * tokens:(f + 1) * tokens] = F.scaled_dot_product_attention(
            qs, ks, vs, scale=scale).permute(1, 0, 2)
    return out


def alpha_fn(down_w, up_w, dt_bias, a_log, num_heads, head_dim):
    """frame_mean [F, hidden] fp32 tensor -> alpha [F, H, d] fp32 tensor through
    oracle.vda.frame_alpha (FrameKDAAlpha, layers.py:36-69, pinned to the reference's
    own output by tests/golden/alpha_golden.npz), from the given weights."""
    w = [np.asarray(t, np.float64) for t in (down_w, up_w, dt_bias, a_log)]

    def fn(frame_mean):
        out = ovda.frame_alpha(frame_mean.double().numpy(), w[0], w[1], w[2], w[3], num_heads, head_dim)
        return torch.from_numpy(out).float()
    return fn


def block_reference(x, temb, w, frames, tokens, cfg, alpha_fn, text_rows=0, out_frames=None):
    """x [text_rows + T, hidden] bf16 values; w: dict of dequantised fp32 weights / biases.

    The attention layout follows cfg.radius / cfg.chunk / cfg.anchor_frames /
    cfg.text_state (defaults: +-radius frames, no anchors, no text seed) with the
    text rows (global, dense) first: window.py:56-111 for the softmax,
    branch.py:256-402 for the linear branch (anchor frames dropped under "both",
    half the prompt state seeding both scans), hybrid_attention.py:200-255 for
    the merge (to_out on every row, to_out_linear on the video rows only, and not
    at all when every window spans the clip).  w["o_b"] is to_out's plus
    to_out_linear's bias; w["o_b_softmax"] (to_out's alone) is needed for text rows
    or a clip-spanning window.

    out_frames (a list of video frame indices): return only those frames' rows, in
    that order (text rows excluded), for checks at full size.  Everything a sampled
    row depends on is still computed for every row (pre-norm, QKV and gates of the
    whole sequence: the softmax keys, the VDA scans and alpha's frame means), while
    the window softmax, the output projection and the FFN run on the sampled rows
    only.
    """
    from . import window as owin
    hd, H, d = cfg.hidden, cfg.heads, cfg.head_dim
    chunk = getattr(cfg, "chunk", 0)
    anchors = getattr(cfg, "anchor_frames", "none")
    L = text_rows
    T = frames * tokens
    n = L + T
    x = x.float()
    # The eager bf16 AdaLN: SiLU of the bf16 embedding is itself a bf16 tensor before the
    # projection (at full size the peaked window softmax turns the 2^-9 difference of
    # skipping that rounding into a few percent of the block output).
    ada = _bf16(_bf16(F.silu(_bf16(temb.float()))) @ w["adaln_w"].T + w["adaln_b"]).view(6, hd)
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = ada
    y1 = prenorm(x, w["norm1"], scale_msa, shift_msa, cfg.eps)
    qkv = _linear(_qdq(y1), w["qkv"], w["qkv_b"])
    q, k, v = (qkv[:, i * hd:(i + 1) * hd].reshape(n, H, d) for i in range(3))
    sgate = _bf16(torch.sigmoid(_bf16(y1 @ w["sg_w"].T + w["sg_b"])))
    beta = _bf16(torch.sigmoid(_bf16(y1 @ w["beta_w"].T)))
    lg = _bf16(torch.sigmoid(_bf16(_bf16(y1 @ w["og_down"].T) @ w["og_up"].T + w["og_b"])))
    bounds = owin.window_bounds(frames, cfg.radius, chunk)
    if out_frames is None:
        rows = torch.arange(n)
    else:
        rows = torch.cat([torch.arange(L + f * tokens, L + (f + 1) * tokens) for f in out_frames])
    if L or chunk or anchors != "none":
        att = owin.window_attention(q, k, v, frames, tokens, bounds, d ** -0.5, text_rows=L,
                                    anchor_frames=anchors, only_frames=out_frames)
    else:
        att = window_attention(q, k, v, frames, tokens, cfg.radius, d ** -0.5, only_frames=out_frames)
    att = _bf16(_bf16(att[rows]) * sgate[rows][..., None]).reshape(len(rows), hd)
    video = rows >= L
    o = torch.empty(len(rows), hd)
    if L and out_frames is None:
        o[:L] = _bf16(_bf16(_qdq(att[:L]) @ w["o"].T) + w["o_b_softmax"].float())
    av = _qdq(att[video]) @ w["o"].T
    if owin.full_cover(bounds, frames):
        o[video] = _bf16(_bf16(av) + w["o_b_softmax"].float())
    else:
        frame_mean = y1[L:].view(frames, tokens, hd).mean(1)
        alpha = alpha_fn(frame_mean).numpy()
        seed = None
        if getattr(cfg, "text_state", False) and L:
            seed = ovda.text_seed(k[:L].numpy(), v[:L].numpy(), beta[:L].numpy())
        kw = {} if out_frames is None or anchors == "both" else {"out_frames": out_frames}
        lin = ovda.branch_forward(q[L:].numpy(), k[L:].numpy(), v[L:].numpy(), beta[L:].numpy(),
                                  lg[L:].view(T, H, d).numpy(), alpha, bounds, frames, tokens,
                                  skip_ends=anchors == "both", seed=seed, **kw)
        lin = torch.from_numpy(lin)[rows[video] - L]
        o[video] = _bf16(_bf16(av + _qdq(lin) @ w["ol"].T) + w["o_b"].float())
    xr = x[rows]
    x1 = _bf16(xr + _bf16(gate_msa * o))
    y2 = prenorm(x1, w["norm2"], scale_mlp, shift_mlp, cfg.eps)
    up = _linear(_qdq(y2), w["up"], w["up_b"])
    act = _bf16(F.gelu(up, approximate=cfg.gelu))
    down = _linear(_qdq(act), w["down"], w["down_b"])
    return _bf16(x1 + _bf16(gate_mlp * down))
