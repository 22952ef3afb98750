"""numpy restatement of the reference VDA branch (frame-wise bidirectional delta rule).

TEST INFRASTRUCTURE ONLY (see the package docstring).

The eager CPU body of the reference, step by step, with its bf16 rounding
points kept and its fp32 arithmetic carried in ``acc`` precision (fp64 by
default, so the oracle is at least as accurate as the path it checks):

  features  SiLU, L2 over d (eps 1e-6) .. src/models/linear_attention/features.py:47-60
  stats     A = sym((k*beta)^T k) fp32,
            B = bf16((bf16(v*beta))^T k) . src/models/linear_attention/scan.py:238-267
  factor    T = diag(alpha)(I+A)^-1,
            J = B (I+A)^-1 .............. src/models/linear_attention/delta_rule.py:45-60
  scans     s_t = s_{t-1} T_t + J_t, fwd and rev,
            start 0 or the text seed .... src/models/linear_attention/scan.py:270-307
  gather    prefix[lo-1]*prod(alpha) +
            suffix[hi+1]*prod(alpha) .... src/models/linear_attention/scan.py:361-496
  readout   einsum fhvk,fshk->fshv (bf16)  src/models/linear_attention/branch.py:470-482
  epilogue  RMSNorm(d) * w, * gate ...... src/models/ops/rms_norm.py:29-32
  text seed 0.5 * B_t (I+A_t)^-1 ........ src/models/linear_attention/branch.py:190-238
  anchors   skip_ends slicing/rebase .... src/models/linear_attention/branch.py:380-401
  alpha     FrameKDAAlpha ............... src/models/linear_attention/layers.py:36-69
  bounds    window_bounds ............... src/models/softmax_attention/window.py:26-52
"""
from __future__ import annotations

import numpy as np

from .mxfp8 import round_bf16


def window_bounds(num_frames: int, radius: int, chunk: int = 0):
    if chunk <= 0:
        return [(t - radius, t + radius) for t in range(num_frames)]
    return [(((t // chunk) - radius) * chunk, ((t // chunk) + radius + 1) * chunk - 1)
            for t in range(num_frames)]


def silu(x, acc=np.float32):
    x = np.asarray(x, dtype=acc)
    return x / (1.0 + np.exp(-x))


def features(raw, l2norm: bool):
    """[N, H, d] bf16 values (as fp32) -> bf16 features (as fp32).

    The eager body's SiLU then L2 normalisation over d (eps 1e-6), evaluated as the
    reference evaluates it (_activate_body, features.py:47-60): torch CPU silu and
    normalize on the bf16 tensor, so every rounding point (bf16 silu, bf16 norm,
    bf16 quotient) is torch's own; multithreaded, which keeps full-size checks fast."""
    import torch
    import torch.nn.functional as Fn
    x = Fn.silu(torch.from_numpy(np.ascontiguousarray(raw, np.float32)).to(torch.bfloat16))
    if l2norm:
        x = Fn.normalize(x, dim=-1, eps=1e-6).to(x.dtype)
    return x.float().numpy()


def frame_statistics(k, v, beta, acc=np.float64):
    """k, v [F, H, S, d] bf16 features; beta [F, H, S] bf16 -> A, B [F, H, d, d]."""
    k = np.asarray(k, acc)
    kb = k * np.asarray(beta, acc)[..., None]
    a = np.matmul(np.swapaxes(kb, -1, -2), k)
    a = 0.5 * (a + np.swapaxes(a, -1, -2))
    vb = round_bf16(np.asarray(v, np.float32) * np.asarray(beta, np.float32)[..., None])
    b = np.matmul(np.swapaxes(np.asarray(vb, acc), -1, -2), k)
    return a, round_bf16(b.astype(np.float32)).astype(acc)


def delta_factors(a, b, alpha=None):
    """T = diag(alpha) (I + A)^-1 and J = B (I + A)^-1, per trailing 128x128 pair."""
    d = a.shape[-1]
    inv = np.linalg.inv(np.eye(d) + np.asarray(a, np.float64))
    t = inv if alpha is None else np.asarray(alpha, np.float64)[..., :, None] * inv
    return t, np.asarray(b, np.float64) @ inv


def run_scans(t, j, seed=None):
    """Forward and reverse state banks, [F, H, d, d] each."""
    f = t.shape[0]
    start = np.zeros_like(j[0]) if seed is None else np.asarray(seed, j.dtype)
    prefix = np.empty_like(j)
    suffix = np.empty_like(j)
    state = start
    for i in range(f):
        state = state @ t[i] + j[i]
        prefix[i] = state
    state = start
    for i in range(f - 1, -1, -1):
        state = state @ t[i] + j[i]
        suffix[i] = state
    return prefix, suffix


def gather(prefix, suffix, alpha, bounds, seed=None, bridge=True):
    """State outside each frame's window, decayed into that frame. [F, H, d, d]."""
    f = prefix.shape[0]
    alpha = np.maximum(np.asarray(alpha, np.float64), 1e-12)
    start = np.zeros_like(prefix[0]) if seed is None else np.asarray(seed, prefix.dtype)
    out = np.empty_like(prefix)
    for t, (lo, hi) in enumerate(bounds):
        left = prefix[lo - 1] if lo > 0 else (start if seed is not None else 0 * start)
        right = suffix[hi + 1] if hi + 1 < f else (start if seed is not None else 0 * start)
        if bridge:
            left = left * alpha[max(0, lo):t + 1].prod(0)[..., None, :]
            right = right * alpha[t:min(f, hi + 1)].prod(0)[..., None, :]
        out[t] = left + right
    return out


def rms_gate_epilogue(readout, weight, gate, eps=1e-6):
    """Eager RMSNorm(d) * w then * gate, bf16 rounding after every op."""
    r = np.asarray(readout, np.float32)
    ms = (r.astype(np.float64) ** 2).sum(-1, keepdims=True) / r.shape[-1]
    inv = round_bf16((1.0 / np.sqrt(ms + eps)).astype(np.float32))
    y = round_bf16(r * inv)
    y = round_bf16(y * round_bf16(np.asarray(weight, np.float32)))
    return round_bf16(y * np.asarray(gate, np.float32))


def text_seed(tk_raw, tv_raw, t_beta, scale=0.5):
    """0.5 * S_text: the prompt written into a zero state as one chunk. [H, d, d]."""
    length, h, d = tk_raw.shape
    k = features(tk_raw, True).reshape(1, length, h, d).transpose(0, 2, 1, 3)
    v = features(tv_raw, False).reshape(1, length, h, d).transpose(0, 2, 1, 3)
    beta = np.asarray(t_beta, np.float32).reshape(1, length, h).transpose(0, 2, 1)
    a, b = frame_statistics(k, v, beta)
    _, inj = delta_factors(a, b)
    return scale * inj[0]


def readout(q_raw, k_raw, v_raw, beta, gate, alpha, bounds, num_frames, tokens_per_frame,
            norm_weight=None, eps=1e-6, seed=None, bridge=True, return_parts=False, out_frames=None):
    """The branch body over the frames it owns. Returns [F*S, H*d] (fp32 of bf16).

    q_raw/k_raw/v_raw [F*S, H, d] and gate [F*S, H, d] hold bf16 values, beta
    [F*S, H] bf16 values, alpha [F, H, d] fp32, seed [H, d, d] or None.
    out_frames: read out only those frames (their rows; the other rows are zero);
    the statistics, factors and scans still cover every frame.
    """
    f, s = num_frames, tokens_per_frame
    n, h, d = q_raw.shape
    assert n == f * s
    if out_frames is not None:
        return _readout_frames(q_raw, k_raw, v_raw, beta, gate, alpha, bounds, f, s, norm_weight,
                               eps, seed, bridge, out_frames)
    q = features(q_raw, True).reshape(f, s, h, d)
    k = features(k_raw, True).reshape(f, s, h, d).transpose(0, 2, 1, 3)
    v = features(v_raw, False).reshape(f, s, h, d).transpose(0, 2, 1, 3)
    b = np.asarray(beta, np.float32).reshape(f, s, h).transpose(0, 2, 1)
    a_stat, b_stat = frame_statistics(k, v, b)
    t, j = delta_factors(a_stat, b_stat, alpha)
    prefix, suffix = run_scans(t, j, seed)
    state = round_bf16(gather(prefix, suffix, alpha, bounds, seed, bridge).astype(np.float32))
    r = np.matmul(q.astype(np.float64).transpose(0, 2, 1, 3),
                  np.swapaxes(state.astype(np.float64), -1, -2))        # [F, H, S, d]
    r = round_bf16(r.transpose(0, 2, 1, 3).astype(np.float32)).reshape(n, h, d)
    w = np.ones(d, np.float32) if norm_weight is None else norm_weight
    out = rms_gate_epilogue(r, w, np.asarray(gate, np.float32).reshape(n, h, d), eps)
    out = out.reshape(n, h * d)
    if return_parts:
        return out, dict(a=a_stat, b=b_stat, t=t, j=j, prefix=prefix, suffix=suffix,
                         state=state, readout=r)
    return out


def _readout_frames(q_raw, k_raw, v_raw, beta, gate, alpha, bounds, f, s, norm_weight, eps, seed,
                    bridge, out_frames):
    n, h, d = q_raw.shape
    k = features(k_raw, True).reshape(f, s, h, d).transpose(0, 2, 1, 3)
    v = features(v_raw, False).reshape(f, s, h, d).transpose(0, 2, 1, 3)
    b = np.asarray(beta, np.float32).reshape(f, s, h).transpose(0, 2, 1)
    a_stat, b_stat = frame_statistics(k, v, b)
    t, j = delta_factors(a_stat, b_stat, alpha)
    prefix, suffix = run_scans(t, j, seed)
    state = round_bf16(gather(prefix, suffix, alpha, bounds, seed, bridge).astype(np.float32))
    w = np.ones(d, np.float32) if norm_weight is None else norm_weight
    out = np.zeros((n, h * d), np.float32)
    for fr in out_frames:
        rows = slice(fr * s, (fr + 1) * s)
        q = features(q_raw[rows], True)                                  # [S, H, d]
        r = np.matmul(q.astype(np.float64).transpose(1, 0, 2),
                      np.swapaxes(state[fr].astype(np.float64), -1, -2))  # [H, S, d]
        r = round_bf16(r.transpose(1, 0, 2).astype(np.float32))
        g = np.asarray(gate[rows], np.float32)
        out[rows] = rms_gate_epilogue(r, w, g, eps).reshape(s, h * d)
    return out


def branch_forward(q_raw, k_raw, v_raw, beta, gate, alpha, bounds, num_frames,
                   tokens_per_frame, skip_ends=False, **kw):
    """Module-level routing: anchor frames dropped from the input and zeroed."""
    f, s = num_frames, tokens_per_frame
    n, h, d = q_raw.shape
    if not skip_ends:
        return readout(q_raw, k_raw, v_raw, beta, gate, alpha, bounds, f, s, **kw)
    out = np.zeros((n, h * d), np.float32)
    if f <= 2:
        return out
    inner = slice(s, (f - 1) * s)
    out[inner] = readout(q_raw[inner], k_raw[inner], v_raw[inner], beta[inner], gate[inner],
                         alpha[1:-1], [(lo - 1, hi - 1) for lo, hi in bounds[1:f - 1]],
                         f - 2, s, **kw)
    return out


def softplus(x):
    x = np.asarray(x, np.float64)
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20))))


def frame_alpha(frame_mean, down_w, up_w, dt_bias, a_log, num_heads, head_dim):
    """FrameKDAAlpha: exp(-exp(A_log) * softplus(up(down(mean)) + dt_bias)). [F, H, d]."""
    delta = np.asarray(frame_mean, np.float64) @ np.asarray(down_w, np.float64).T
    delta = delta @ np.asarray(up_w, np.float64).T + np.asarray(dt_bias, np.float64)
    scale = np.exp(np.asarray(a_log, np.float64))[:, None]
    delta = delta.reshape(-1, num_heads, head_dim)
    return np.exp(-scale * softplus(delta))
