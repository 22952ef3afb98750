"""CPU restatement of the window softmax with global (text) rows and anchor frames.
TEST INFRASTRUCTURE ONLY.

Reference: ec-jt/vdn src/models/softmax_attention/window.py:26-52 (window_bounds,
frame and chunk-aligned modes) and :56-111 (window_softmax_reference): exact
softmax in which (video, video) pairs are limited to the query frame's window
while every pair that involves a global (text) row stays dense in both
directions; anchor "rows" make frames 0 and F-1 attend to every video frame,
anchor "columns" add frames 0 and F-1 to every video query's keys (once: a frame
already inside the window is not repeated).  Sequence layout: `text_rows` global
rows first, then F * S video rows, frame-major.  Pinned by
tests/golden/window_golden.npz (the reference function run on CPU).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

ANCHOR_MODES = ("none", "columns", "rows", "both")


def window_bounds(num_frames, radius, chunk=0):
    """Per-frame inclusive [lo, hi], unclamped (window.py:26-52)."""
    if chunk <= 0:
        return [(t - radius, t + radius) for t in range(num_frames)]
    return [((t // chunk - radius) * chunk, (t // chunk + radius + 1) * chunk - 1)
            for t in range(num_frames)]


def frame_keys(bounds, num_frames, anchor_frames="none"):
    """Per query frame: (lo, hi) clamped window and the extra anchor key frames."""
    if anchor_frames not in ANCHOR_MODES:
        raise ValueError(f"anchor_frames must be one of {ANCHOR_MODES}")
    out = []
    for f in range(num_frames):
        lo, hi = max(bounds[f][0], 0), min(bounds[f][1], num_frames - 1)
        if anchor_frames in ("rows", "both") and f in (0, num_frames - 1):
            lo, hi = 0, num_frames - 1
        extra = []
        if anchor_frames in ("columns", "both"):
            for a in (0, num_frames - 1):
                if not lo <= a <= hi and a not in extra:
                    extra.append(a)
        out.append((lo, hi, extra))
    return out


def _sdpa(q, k, v, scale):
    """[rows, H, d] queries over [keys, H, d] -> [rows, H, d], fp32 dense softmax."""
    o = F.scaled_dot_product_attention(q.permute(1, 0, 2)[None], k.permute(1, 0, 2)[None],
                                       v.permute(1, 0, 2)[None], scale=scale)
    return o[0].permute(1, 0, 2)


def window_attention(q, k, v, num_frames, tokens_per_frame, bounds, scale, text_rows=0,
                     anchor_frames="none", only_frames=None):
    """q/k/v [text_rows + F*S, H, d] (fp32 values) -> [same] fp32.  only_frames: compute
    those video query frames only (text rows and other frames are left zero)."""
    q, k, v = q.float(), k.float(), v.float()
    L, S = text_rows, tokens_per_frame
    out = torch.zeros_like(q)
    if L and only_frames is None:
        out[:L] = _sdpa(q[:L], k, v, scale)
    gk, gv = k[:L], v[:L]
    for f, (lo, hi, extra) in enumerate(frame_keys(bounds, num_frames, anchor_frames)):
        if only_frames is not None and f not in only_frames:
            continue
        keys = [gk, k[L + lo * S:L + (hi + 1) * S]] + [k[L + a * S:L + (a + 1) * S] for a in extra]
        vals = [gv, v[L + lo * S:L + (hi + 1) * S]] + [v[L + a * S:L + (a + 1) * S] for a in extra]
        r0 = L + f * S
        out[r0:r0 + S] = _sdpa(q[r0:r0 + S], torch.cat(keys), torch.cat(vals), scale)
    return out


def full_cover(bounds, num_frames):
    """Every frame's window spans the clip: the linear branch has nothing to add."""
    return all(lo <= 0 and hi >= num_frames - 1 for lo, hi in bounds)
