"""A stack of hybrid blocks and the denoise loop around it.

The reference runs its 40-block H3 transformer once per denoising step over the
packed sequence [text rows | video rows] (src/inference/utils/ulysses.py:601-714
for the sharded transformer forward, the text rows packed first as global rows).
Here the stack works in the blocks' hidden space: the per-step text conditioning
is packed in front of the current video rows, every block runs (text rows dense
in the softmax, video rows in their window, the VDA branch over the video rows),
and an Euler update moves the video rows by the stack's output.  Patch embedding,
output projection and the sampler's schedule are outside the hot path.
"""
from __future__ import annotations

import torch
from torch import nn

from .block import BlockConfig, HybridBlock

__all__ = ["HybridStack", "denoise", "local_rows"]


class HybridStack(nn.Module):
    def __init__(self, cfg: BlockConfig | None = None, depth=40, *, seed=0, device="cuda", init="host"):
        super().__init__()
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.cfg = cfg or BlockConfig()
        self.blocks = nn.ModuleList(HybridBlock(self.cfg, seed=seed + 7919 * i, device=device, init=init)
                                    for i in range(depth))

    @property
    def transformer_blocks(self) -> nn.ModuleList:
        """The reference model's name for its block list (install_ulysses walks it)."""
        return self.blocks

    @torch.no_grad()
    def forward(self, x, temb, frames, tokens, runtime=None, text_rows=0):
        for block in self.blocks:
            x = block(x, temb, frames, tokens, runtime, text_rows=text_rows)
        return x


def local_rows(text_rows, runtime=None, total=None):
    """(text, video) row ranges of this rank's shard of the packed sequence [text | video]:
    text rows [a, b) of the context and video rows [c, e) of the clip."""
    if runtime is None or runtime.world_size == 1:
        return (0, text_rows), (0, total - text_rows)
    lo, hi = runtime.local_start, runtime.local_end
    t = (min(lo, text_rows), min(hi, text_rows))
    v = (max(lo, text_rows) - text_rows, max(hi, text_rows) - text_rows)
    return t, v


@torch.no_grad()
def denoise(stack: HybridStack, video, text, tembs, frames, tokens, *, packed=None, dt=None,
            runtime=None):
    """Euler loop: for each step i, packed = [text_i | video]; video += dt * stack(packed)[video rows]
    with dt = -1 / steps unless given.  text [steps, L, hidden] or [L, hidden] (the same
    context every step) or None; tembs [steps, hidden].  video is updated in place and
    returned: all F*S rows, or with a Ulysses runtime (configured for L + F*S rows) this
    rank's video rows of the sharded packed sequence."""
    steps = tembs.shape[0]
    L = 0 if text is None else text.shape[-2]
    if runtime is not None and runtime.world_size > 1:
        (ta, tb), (va, vb) = local_rows(L, runtime)
        if runtime.sequence_length != L + frames * tokens or video.shape[0] != vb - va:
            raise ValueError("video must hold this rank's video rows of the configured sequence")
    else:
        (ta, tb), (va, vb) = local_rows(L, None, L + video.shape[0])
    nt = tb - ta
    n = nt + video.shape[0]
    if packed is None:
        packed = torch.empty(n, video.shape[1], device=video.device, dtype=video.dtype)
    dt = -1.0 / steps if dt is None else dt
    for i in range(steps):
        if nt:
            packed[:nt].copy_((text[i] if text.dim() == 3 else text)[ta:tb])
        packed[nt:].copy_(video)
        out = stack(packed, tembs[i], frames, tokens, runtime, text_rows=L)
        video.add_(out[nt:], alpha=dt)
    return video
