"""CPU restatement of the linear branch's separable short conv. TEST INFRASTRUCTURE ONLY.

Reference: ec-jt/vdn src/models/linear_attention/features.py:133-209
(LinearAttentionSepConv: depthwise 5x5 SPATIAL conv per frame, then a depthwise
5-tap TEMPORAL conv across frames, both bias-free, zero padding) and :12-40
(_temporal_shift / _temporal_conv), followed by the features SiLU [-> L2Norm]
(features.py:47-60).  Pinned by tests/golden/sepconv_golden.npz (the reference
run on CPU).

Rounding points: the spatial half is one bf16 rounding of an exact sum (the
reference's conv2d produces a bf16 tensor); the temporal half has two forms,
`temporal_eager` (each product and each partial sum rounded to bf16, the eager
CPU shift) and `temporal` (one rounding of an exact sum: the fused form, which
the reference's compiled CUDA path and this repository's kernel compute).
"""
from __future__ import annotations

import numpy as np

from .mxfp8 import round_bf16

KERNEL = 5


def spatial(x, w_sp, num_frames, frame_size):
    """x [F*S, C] bf16 values; w_sp [C, 5, 5] -> [F, S, C] bf16 values (exact sum, one rounding)."""
    gh, gw = frame_size
    c = x.shape[-1]
    vol = np.asarray(x, np.float64).reshape(num_frames, gh, gw, c)
    pad = np.zeros((num_frames, gh + 4, gw + 4, c))
    pad[:, 2:2 + gh, 2:2 + gw] = vol
    w = np.asarray(w_sp, np.float64).reshape(c, 5, 5)
    out = np.zeros((num_frames, gh, gw, c))
    for dy in range(KERNEL):
        for dx in range(KERNEL):
            out += pad[:, dy:dy + gh, dx:dx + gw, :] * w[:, dy, dx]
    return round_bf16(out.astype(np.float32)).reshape(num_frames, gh * gw, c)


def temporal(s, w_tm):
    """s [F, S, C] bf16 values; w_tm [C, 5] -> [F, S, C]: one rounding of the exact 5-tap sum."""
    f = s.shape[0]
    sp = np.zeros((f + 4,) + s.shape[1:])
    sp[2:2 + f] = np.asarray(s, np.float64)
    w = np.asarray(w_tm, np.float64)
    out = np.zeros(s.shape)
    for dt in range(KERNEL):
        out += sp[dt:dt + f] * w[:, dt]
    return round_bf16(out.astype(np.float32))


def temporal_eager(s, w_tm):
    """The eager shift (features.py:12-31): bf16 product, bf16 running sum, taps in order."""
    f = s.shape[0]
    sp = np.zeros((f + 4,) + s.shape[1:], np.float32)
    sp[2:2 + f] = np.asarray(s, np.float32)
    w = np.asarray(w_tm, np.float32)
    out = None
    for dt in range(KERNEL):
        part = round_bf16(sp[dt:dt + f] * w[:, dt])
        out = part if out is None else round_bf16(out + part)
    return out


def conv_features(tokens, w_sp, w_tm, num_frames, frame_size, l2norm, eager=False):
    """[F*S, H, d] raw projection -> conv -> SiLU [-> L2Norm] features, [F*S, H, d]."""
    from .vda import features
    n, h, d = tokens.shape
    s = spatial(tokens.reshape(n, h * d), w_sp, num_frames, frame_size)
    t = (temporal_eager if eager else temporal)(s, w_tm)
    return features(t.reshape(n, h, d), l2norm)
