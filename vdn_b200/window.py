"""The block's window-softmax branch: dense legs on the library kernel, merged natively.

The frame window [t - r, t + r] is the union of 2r + 1 dense attentions (query
frame t against key frame t + delta), each one batched cuDNN SDPA call over all
frames with no key/value duplication (the reference's own dense leg on B200 is
cuDNN too: src/models/softmax_attention/decomposed.py).  vdn_window_merge then
combines the legs by their log-sum-exps, applies the softmax gate and writes
bf16 and/or MXFP8.  The attention kernel itself is library code and outside the
parity contract; it is counted in block timings only.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

__all__ = ["window_softmax"]


def _legs(q, k, v, frames, tokens, radius, scale):
    """Per delta: (out [rows, H*d] bf16, lse [batches, H, S] fp32, batch0, frame_lo, frame_hi)."""
    t, h, d = q.shape
    qb = q.view(frames, tokens, h, d).permute(0, 2, 1, 3)
    kb = k.view(frames, tokens, h, d).permute(0, 2, 1, 3)
    vb = v.view(frames, tokens, h, d).permute(0, 2, 1, 3)
    legs = []
    for delta in range(-radius, radius + 1):
        lo, hi = max(0, -delta), min(frames, frames - delta)   # query frames [lo, hi)
        if hi <= lo:
            continue
        out, lse = torch.ops.aten._scaled_dot_product_cudnn_attention(
            qb[lo:hi], kb[lo + delta:hi + delta], vb[lo + delta:hi + delta], None, True, 0.0,
            False, False, scale=scale)[:2]
        # cuDNN returns token-major storage ([B, S, H, d] memory) and lse [B, H, S, 1].
        if out.stride(2) != h * d or out.stride(1) != d:
            out = out.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
        legs.append((out, lse.contiguous(), lo, lo, hi - 1))
    return legs


def window_softmax(q, k, v, gate, frames, tokens, radius=1, scale=None, *, out=None,
                   quantize=False):
    """Gated window softmax over [F*S, H, d] q / k / v views (last dim contiguous).

    gate [F*S, H] bf16.  Writes bf16 into `out` ([F*S, H, >= d] view, last dim
    contiguous) when given and returns MXFP8 (codes, scales) of the gated output
    when quantize=True.
    """
    t, h, d = q.shape
    if t != frames * tokens:
        raise ValueError("q must hold frames * tokens rows")
    if radius < 0 or 2 * radius + 1 > 5:
        raise ValueError("window radius must lie in [0, 2]")
    scale = d ** -0.5 if scale is None else scale
    legs = _legs(q, k, v, frames, tokens, radius, scale)
    n = len(legs)
    outs = (C.c_void_p * n)(*[x[0].data_ptr() for x in legs])
    lses = (C.c_void_p * n)(*[x[1].data_ptr() for x in legs])
    b0 = (C.c_int * n)(*[x[2] for x in legs])
    flo = (C.c_int * n)(*[x[3] for x in legs])
    fhi = (C.c_int * n)(*[x[4] for x in legs])
    qc = sc = None
    if quantize:
        rp = (t + 127) // 128 * 128
        qc = torch.empty((rp, h * d), dtype=torch.uint8, device=q.device)
        sc = torch.empty(rp * h * d // 32, dtype=torch.uint8, device=q.device)
    _lib.call("vdn_window_merge", n, outs, lses, b0, flo, fhi, frames, tokens, h, d,
              _lib.ptr(gate), gate.stride(0), gate.stride(1), _lib.ptr(out),
              out.stride(0) if out is not None else 0, out.stride(1) if out is not None else 0,
              _lib.ptr(qc), _lib.ptr(sc), _lib.stream_of(q.device))
    return (qc, sc) if quantize else None
