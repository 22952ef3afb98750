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

__all__ = ["HybridStack", "denoise"]


class HybridStack(nn.Module):
    def __init__(self, cfg: BlockConfig | None = None, depth=40, *, seed=0, device="cuda", init="host"):
        super().__init__()
        if depth < 1:
            raise ValueError("depth must be >= 1")
        self.cfg = cfg or BlockConfig()
        self.blocks = nn.ModuleList(HybridBlock(self.cfg, seed=seed + 7919 * i, device=device, init=init)
                                    for i in range(depth))

    @torch.no_grad()
    def forward(self, x, temb, frames, tokens, runtime=None, text_rows=0):
        for block in self.blocks:
            x = block(x, temb, frames, tokens, runtime, text_rows=text_rows)
        return x


@torch.no_grad()
def denoise(stack: HybridStack, video, text, tembs, frames, tokens, *, packed=None, dt=None):
    """Euler loop: for each step i, packed = [text_i | video]; video += dt * stack(packed)[video rows]
    with dt = -1 / steps unless given.  video [F*S, hidden] bf16 (updated in place and
    returned); text [steps, L, hidden] or [L, hidden] (the same context every step) or
    None; tembs [steps, hidden]."""
    steps = tembs.shape[0]
    L = 0 if text is None else text.shape[-2]
    n = L + video.shape[0]
    if packed is None:
        packed = torch.empty(n, video.shape[1], device=video.device, dtype=video.dtype)
    dt = -1.0 / steps if dt is None else dt
    for i in range(steps):
        if L:
            packed[:L].copy_(text[i] if text.dim() == 3 else text)
        packed[L:].copy_(video)
        out = stack(packed, tembs[i], frames, tokens, text_rows=L)
        video.add_(out[L:], alpha=dt)
    return video
