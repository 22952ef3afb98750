"""The linear branch's separable short conv on the library kernel.

Mirrors ec-jt/vdn src/models/linear_attention/features.py:133-209
(LinearAttentionSepConv): per convolved projection a depthwise 5x5 spatial conv
per frame and a depthwise 5-tap temporal conv across frames, bias-free, zero
padded, with the same parameter names and shapes (`{proj}_sp` Conv2d [C,1,5,5],
`{proj}_tm` Conv1d [C,1,5]) and initialisation, so checkpoints load unchanged.
`apply` returns the conv output (bf16); the branch's SiLU [-> L2Norm] then runs
inside the statistics / readout kernels exactly as for unconvolved projections.
Inference only; no PyTorch fallback for the conv itself.
"""
from __future__ import annotations

import torch
from torch import nn

from . import _lib

__all__ = ["LinearAttentionSepConv", "sepconv"]

SHORT_CONV_TARGETS = ("q", "k", "v")


def sepconv(tokens: torch.Tensor, num_frames: int, frame_size, w_spatial: torch.Tensor,
            w_temporal: torch.Tensor) -> torch.Tensor:
    """[F*S, H, d] bf16 (or [F*S, C]) -> conv output, same shape, contiguous.

    w_spatial [C, 1, 5, 5] / [C, 25], w_temporal [C, 1, 5] / [C, 5] (any float dtype;
    rounded to bf16 like the reference's bf16 module weights).
    """
    if tokens.dtype != torch.bfloat16 or not tokens.is_cuda or tokens.stride(-1) != 1:
        raise ValueError("short conv needs CUDA bf16 tokens with a contiguous last dimension")
    _lib.require_device(tokens, "tokens")
    gh, gw = frame_size
    n = tokens.shape[0]
    if n != num_frames * gh * gw:
        raise ValueError(f"{n} rows != num_frames * height * width = {num_frames * gh * gw}")
    flat = tokens.reshape(n, -1) if tokens.ndim == 3 else tokens
    if flat.stride(-1) != 1:
        flat = flat.contiguous()
    c = flat.shape[1]
    wsp = w_spatial.reshape(c, 25).to(torch.bfloat16).t().contiguous()      # [25, C]
    wtm = w_temporal.reshape(c, 5).to(torch.bfloat16).t().contiguous()      # [5, C]
    out = torch.empty(n, c, device=tokens.device, dtype=torch.bfloat16)
    scratch = torch.empty(n, c, device=tokens.device, dtype=torch.bfloat16)
    _lib.call("vdn_sepconv", _lib.ptr(flat), flat.stride(0), num_frames, gh, gw, c, _lib.ptr(wsp),
              _lib.ptr(wtm), _lib.ptr(scratch), _lib.ptr(out), c, _lib.stream_of(tokens.device))
    return out.view(tokens.shape)


class LinearAttentionSepConv(nn.Module):
    """Depthwise short conv on the projections named in `projs` (features.py:133-209)."""

    KERNEL = 5

    def __init__(self, channels, projs=("k", "v")):
        super().__init__()
        projs = tuple(projs)
        if any(p not in SHORT_CONV_TARGETS for p in projs) or len(set(projs)) != len(projs):
            raise ValueError(f"projs={projs!r}; expected a distinct subset of {SHORT_CONV_TARGETS}")
        self.projs = projs
        k = self.KERNEL
        for name in self.projs:
            sp = nn.Conv2d(channels, channels, k, padding=k // 2, groups=channels, bias=False)
            nn.init.normal_(sp.weight, std=(k * k) ** -0.5)
            tm = nn.Conv1d(channels, channels, k, padding=k // 2, groups=channels, bias=False)
            nn.init.normal_(tm.weight, std=k ** -0.5)
            setattr(self, f"{name}_sp", sp)
            setattr(self, f"{name}_tm", tm)

    def apply(self, proj, tokens, num_frames, frame_size, heads=None):
        """Conv output of one projection [F*S, H_local, d]; `heads` selects a head range
        (the weights' matching channel slice), unlisted projections pass through."""
        if proj not in self.projs:
            return tokens
        w_sp = getattr(self, f"{proj}_sp").weight
        w_tm = getattr(self, f"{proj}_tm").weight
        if heads is not None:
            d = tokens.shape[-1]
            ch = slice(heads.start * d, heads.stop * d)
            w_sp, w_tm = w_sp[ch], w_tm[ch]
        return sepconv(tokens, num_frames, frame_size, w_sp, w_tm)

    def forward(self, q_raw, k_raw, v_raw, num_frames, frame_size):
        return (self.apply("q", q_raw, num_frames, frame_size),
                self.apply("k", k_raw, num_frames, frame_size),
                self.apply("v", v_raw, num_frames, frame_size))
