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

__all__ = ["window_softmax", "frame_windows", "ANCHOR_MODES"]


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


ANCHOR_MODES = ("none", "columns", "rows", "both")
_MAX_PARTIALS = 5          # partials one vdn_window_merge launch combines


def frame_windows(bounds, frames, anchor_frames="none"):
    """Per query frame (lo, hi, extra): the clamped key-frame window and the anchor
    key frames outside it (window.py:78-101: anchor ROWS make frames 0 and F-1
    dense over the clip, anchor COLUMNS add frames 0 and F-1 to every query once)."""
    if anchor_frames not in ANCHOR_MODES:
        raise ValueError(f"anchor_frames must be one of {ANCHOR_MODES}, got {anchor_frames!r}")
    if len(bounds) != frames:
        raise ValueError("one (lo, hi) window per frame")
    out = []
    for f, (lo, hi) in enumerate(bounds):
        lo, hi = max(int(lo), 0), min(int(hi), frames - 1)
        if lo > hi:
            raise ValueError(f"frame {f}'s window [{lo}, {hi}] is empty inside the clip")
        if anchor_frames in ("rows", "both") and f in (0, frames - 1):
            lo, hi = 0, frames - 1
        extra = []
        if anchor_frames in ("columns", "both"):
            extra = [a for a in dict.fromkeys((0, frames - 1)) if not lo <= a <= hi]
        out.append((lo, hi, extra))
    return out


def _attend(qv, kv, vv, scale):
    """One cuDNN call on [B, H, Sq, d] / [B, H, Sk, d] views -> (out with token-major
    memory [B, Sq, H, d], lse [B, H, Sq])."""
    h, d = qv.shape[1], qv.shape[3]
    o, lse = torch.ops.aten._scaled_dot_product_cudnn_attention(
        qv, kv, vv, None, True, 0.0, False, False, scale=scale)[:2]
    if o.stride(2) != h * d or o.stride(1) != d:
        o = o.permute(0, 2, 1, 3).contiguous().permute(0, 2, 1, 3)
    return o, lse.reshape(qv.shape[0], h, qv.shape[2])


def _rows(t, a, b):
    """Rows [a, b) of a [rows, H, d] tensor as a [1, H, b - a, d] attention operand."""
    return t[a:b].unsqueeze(0).permute(0, 2, 1, 3)


def _flat_leg(qv, kv, vv, tokens, f0, nq, scale):
    """Query frames [f0, f0 + nq) as ONE sequence against the given keys, returned in
    the merge's per-frame layout: out [nq * S, H, d] rows and lse [nq, H, S]."""
    o, lse = _attend(qv, kv, vv, scale)
    h = qv.shape[1]
    lse = lse.reshape(h, nq, tokens).transpose(0, 1).contiguous()
    return (o, lse, f0, f0, f0 + nq - 1)


def _runs(frames_with_key):
    """Consecutive runs [(first, last)] of a sorted frame list, split where `key` changes."""
    runs = []
    for f, key in frames_with_key:
        if runs and runs[-1][1] == f - 1 and runs[-1][2] == key:
            runs[-1][1] = f
        else:
            runs.append([f, f, key])
    return runs


def _general_legs(q, k, v, frames, tokens, text_rows, windows, radius, scale):
    """Partials for the video queries: window legs (one strided batched call for the
    uniform interior of a frame window, one flat call per run of frames sharing a
    window), one leg against the text keys, one per run of frames that add an anchor
    frame as extra keys."""
    L, S = text_rows, tokens
    qv_, kv_, vv_ = q[L:], k[L:], v[L:]
    legs = []
    interior = set()
    if radius is not None:
        interior = {f for f, (lo, hi, _) in enumerate(windows)
                    if (lo, hi) == (f - radius, f + radius)}
        if interior:
            f0, f1 = min(interior), max(interior)
            if interior != set(range(f0, f1 + 1)):
                interior = set()
    if interior:
        f0, n = min(interior), len(interior)
        s0, s1 = qv_.stride(0), qv_.stride(1)
        qb = qv_.as_strided((n, S, qv_.shape[1], qv_.shape[2]), (S * s0, s0, s1, 1),
                            qv_.storage_offset() + f0 * S * s0).permute(0, 2, 1, 3)
        span = 2 * radius + 1
        kvb = []
        for x in (kv_, vv_):
            s0, s1 = x.stride(0), x.stride(1)
            kvb.append(x.as_strided((n, span * S, x.shape[1], x.shape[2]), (S * s0, s0, s1, 1),
                                    x.storage_offset() + (f0 - radius) * S * s0).permute(0, 2, 1, 3))
        o, lse = _attend(qb, kvb[0], kvb[1], scale)
        legs.append((o, lse.contiguous(), f0, f0, f0 + n - 1))
    rest = [(f, (lo, hi)) for f, (lo, hi, _) in enumerate(windows) if f not in interior]
    for a, b, (lo, hi) in _runs(rest):
        legs.append(_flat_leg(_rows(qv_, a * S, (b + 1) * S), _rows(kv_, lo * S, (hi + 1) * S),
                              _rows(vv_, lo * S, (hi + 1) * S), S, a, b - a + 1, scale))
    if L:
        legs.append(_flat_leg(_rows(qv_, 0, frames * S), _rows(k, 0, L), _rows(v, 0, L), S, 0, frames,
                              scale))
    for anchor in sorted({a for _, _, extra in windows for a in extra}):
        with_anchor = [(f, 0) for f, (_, _, extra) in enumerate(windows) if anchor in extra]
        for a, b, _ in _runs(with_anchor):
            legs.append(_flat_leg(_rows(qv_, a * S, (b + 1) * S), _rows(kv_, anchor * S, (anchor + 1) * S),
                                  _rows(vv_, anchor * S, (anchor + 1) * S), S, a, b - a + 1, scale))
    return legs


def _merge_groups(legs, frames):
    """Split the frames into consecutive groups that each meet at most _MAX_PARTIALS legs."""
    groups, g0, active = [], 0, []
    for f in range(frames):
        cover = [j for j, leg in enumerate(legs) if leg[3] <= f <= leg[4]]
        merged = active + [j for j in cover if j not in active]
        if len(merged) > _MAX_PARTIALS:
            groups.append((g0, f - 1, active))
            g0, active = f, cover
        else:
            active = merged
    groups.append((g0, frames - 1, active))
    return groups


def _window_softmax_general(q, k, v, gate, frames, tokens, text_rows, windows, radius, scale, out,
                            quantize):
    n, h, d = q.shape
    L, S = text_rows, tokens
    buf = out
    if buf is None or (quantize and (buf.stride(1) != d or buf.stride(0) != h * d)):
        buf = torch.empty(n, h, d, dtype=torch.bfloat16, device=q.device)
    if L:  # global queries: dense over the whole sequence, then the gate
        o, _ = _attend(_rows(q, 0, L), _rows(k, 0, n), _rows(v, 0, n), scale)
        torch.mul(o[0].permute(1, 0, 2), gate[:L, :, None], out=buf[:L, :, :d])
    legs = _general_legs(q, k, v, frames, tokens, L, windows, radius, scale)
    stream = _lib.stream_of(q.device)
    for g0, g1, idx in _merge_groups(legs, frames):
        sel = [legs[j] for j in idx]
        m = len(sel)
        outs = (C.c_void_p * m)(*[x[0].data_ptr() for x in sel])
        lses = (C.c_void_p * m)(*[x[1].data_ptr() for x in sel])
        b0 = (C.c_int * m)(*[x[2] - g0 for x in sel])
        flo = (C.c_int * m)(*[max(x[3], g0) - g0 for x in sel])
        fhi = (C.c_int * m)(*[min(x[4], g1) - g0 for x in sel])
        r0 = L + g0 * S
        _lib.call("vdn_window_merge", m, outs, lses, b0, flo, fhi, g1 - g0 + 1, S, h, d,
                  C.c_void_p(gate[r0:].data_ptr()), gate.stride(0), gate.stride(1),
                  C.c_void_p(buf[r0:].data_ptr()), buf.stride(0), buf.stride(1), None, None, stream)
    if out is not None and buf is not out:
        out[:, :, :d].copy_(buf)
    if quantize:
        from .mxfp8_quant import quantize_activation
        return quantize_activation(buf.view(n, h * d), check_finite=False)
    return None


def window_softmax(q, k, v, gate, frames, tokens, radius=1, scale=None, *, out=None,
                   quantize=False, bounds=None, text_rows=0, anchor_frames="none"):
    """Gated window softmax over [text_rows + F*S, H, d] q / k / v views (last dim
    contiguous): text rows first (dense in both directions), then the video rows,
    frame-major, each query frame attending to its window.

    gate [rows, H] bf16.  Writes bf16 into `out` ([rows, H, >= d] view, last dim
    contiguous) when given and returns MXFP8 (codes, scales) of the gated output
    when quantize=True.  `bounds` (per-frame [lo, hi], unclamped: frame or
    chunk-aligned windows) overrides `radius`; anchor_frames is one of "none",
    "columns", "rows", "both" (src/models/softmax_attention/window.py:56-111).
    """
    t, h, d = q.shape
    if t != text_rows + frames * tokens or text_rows < 0:
        raise ValueError("q must hold text_rows + frames * tokens rows")
    scale = d ** -0.5 if scale is None else scale
    if bounds is not None or text_rows or anchor_frames != "none" or radius > 2:
        if bounds is None:
            if radius < 0:
                raise ValueError("window radius must be >= 0")
            bounds = [(f - radius, f + radius) for f in range(frames)]
        windows = frame_windows(bounds, frames, anchor_frames)
        r = (bounds[0][1] - bounds[0][0]) // 2
        uniform = all((lo, hi) == (f - r, f + r) for f, (lo, hi) in enumerate(bounds))
        return _window_softmax_general(q, k, v, gate, frames, tokens, text_rows, windows,
                                       r if uniform else None, scale, out, quantize)
    if radius < 0:
        raise ValueError("window radius must be >= 0")
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
