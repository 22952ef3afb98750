"""The block's window-softmax branch: dense attention on the library kernel, gated natively.

Query frame t attends to the key frames [t - r, t + r] (clipped at the clip's
ends).  All interior frames share one batched cuDNN SDPA call whose K / V are
overlapping strided views of the token-major tensors (batch stride = one
frame, sequence = 2r + 1 frames: no key/value duplication); each clipped edge
frame is one more call (the reference's own dense attention on B200 is cuDNN
too: src/models/softmax_attention/decomposed.py).  vdn_window_merge then applies
the softmax gate and writes bf16 and/or MXFP8 (its log-sum-exp merge also
combines split key ranges when a caller passes several partials per frame).
The attention kernel itself is library code and outside the parity contract; it
is counted in block timings only.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

__all__ = ["window_softmax"]


def _span(t, tokens, start_frame, nframes):
    """[n, H, nframes * tokens, d] view whose batch b starts at frame start_frame + b
    (windows of consecutive batches overlap: a strided view, no copy)."""
    rows, h, d = t.shape
    s0, s1 = t.stride(0), t.stride(1)
    return t.as_strided((1, nframes * tokens, h, d), (tokens * s0, s0, s1, 1),
                        t.storage_offset() + start_frame * tokens * s0)


def _windows(q, k, v, frames, tokens, radius, scale):
    """Per call: (out, lse, batch0, frame_lo, frame_hi).

    Interior frames (radius <= t < F - radius) see exactly 2r + 1 key frames
    starting at t - r: one batched call whose K / V are strided views with a
    batch stride of one frame over the token-major tensors.  Each edge frame sees
    a clipped window and gets a call of its own.  One softmax per query frame,
    so the merge only applies the gate (every frame has one partial).
    """
    t, h, d = q.shape
    s0q, s1q = q.stride(0), q.stride(1)
    calls = []
    interior = max(0, frames - 2 * radius)
    if interior:
        f0 = radius
        qv = q.as_strided((interior, tokens, h, d), (tokens * s0q, s0q, s1q, 1),
                          q.storage_offset() + f0 * tokens * s0q).permute(0, 2, 1, 3)
        span = 2 * radius + 1
        kv = []
        for x in (k, v):
            s0, s1 = x.stride(0), x.stride(1)
            kv.append(x.as_strided((interior, span * tokens, h, d), (tokens * s0, s0, s1, 1),
                                   x.storage_offset() + (f0 - radius) * tokens * s0).permute(0, 2, 1, 3))
        calls.append((qv, kv[0], kv[1], f0, f0, f0 + interior - 1))
    edges = [f for f in range(frames) if f < radius or f >= frames - radius]
    for f in edges:
        lo, hi = max(0, f - radius), min(frames - 1, f + radius)
        qv = _span(q, tokens, f, 1).permute(0, 2, 1, 3)
        kv = _span(k, tokens, lo, hi - lo + 1).permute(0, 2, 1, 3)
        vv = _span(v, tokens, lo, hi - lo + 1).permute(0, 2, 1, 3)
        calls.append((qv, kv, vv, f, f, f))
    out = []
    for qv, kv, vv, b0, flo, fhi in calls:
        o, lse = torch.ops.aten._scaled_dot_product_cudnn_attention(
            qv, kv, vv, None, True, 0.0, False, False, scale=scale)[:2]
        # cuDNN returns token-major storage ([B, S, H, d] memory) and lse [B, H, S, 1].
        if o.stride(2) != h * d or o.stride(1) != d:
            o = o.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
        out.append((o, lse.contiguous(), b0, flo, fhi))
    return out


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
    legs = _windows(q, k, v, frames, tokens, radius, scale)
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
