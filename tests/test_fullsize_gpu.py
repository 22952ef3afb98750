"""GPU: the hybrid block at the BASELINE sizes against the CPU composition of the
reference pieces, on sampled frames.

Config 3: one block at hidden 5120, 40 x 128 heads, FFN 13824, 21 frames x 1560
tokens (32760 rows), the geometry bench.py times.  Config 4's shape: two stacked
blocks over 512 text rows packed in front of 60 x 1560 video rows (94112 rows);
the second block takes the first block's GPU output as its input, so each block is
checked on its own at full size.

The oracle (oracle/block.py, out_frames=...) evaluates only the sampled frames'
rows of the window softmax, output projection and FFN, but every row of what those
rows depend on: the pre-norm, QKV and gates of the whole sequence (the softmax
keys, the VDA statistics and scans over every frame, alpha's frame means).  Alpha
comes from the block's FrameKDAAlpha weights through the oracle's restatement
(pinned to the reference's FrameKDAAlpha), not from the module under test.
Tolerance: relative L2 < 1e-2 on the sampled rows, the small-shape block bar
(bf16 rounding points and the rare one-code MXFP8 flips they cause).
"""
import pytest
import torch

from oracle import block as oblock
from test_block_gpu import _reference_alpha, _rel, _weights

pytestmark = pytest.mark.gpu


def _rows(out, frames, tokens, text_rows=0):
    return torch.cat([out[text_rows + f * tokens:text_rows + (f + 1) * tokens] for f in frames])


@torch.no_grad()
def test_block_config3_full_size_sampled_frames(cuda):
    from vdn_b200.block import HybridBlock
    block = HybridBlock(seed=0, device=cuda)                  # BlockConfig() = BASELINE config 3
    cfg = block.cfg
    assert (cfg.hidden, cfg.heads, cfg.head_dim, cfg.ffn) == (5120, 40, 128, 13824)
    frames, tokens = 21, 1560
    g = torch.Generator().manual_seed(2024)
    x = torch.randn(frames * tokens, cfg.hidden, generator=g).bfloat16()
    temb = torch.randn(cfg.hidden, generator=g)
    out = block(x.to(cuda), temb.to(cuda), frames, tokens)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(out).all())
    sample = [0, 10, 20]                                      # both edges and the middle
    ref = oblock.block_reference(x, temb, _weights(block), frames, tokens, cfg, _reference_alpha(block),
                                 out_frames=sample)
    got = _rows(out.cpu(), sample, tokens)
    err = _rel(got.float(), ref)
    assert err < 1e-2, err


@torch.no_grad()
def test_stack_config4_shape_two_blocks_sampled_frames(cuda):
    from vdn_b200.stack import HybridStack
    stack = HybridStack(depth=2, seed=0, device=cuda)
    cfg = stack.cfg
    frames, tokens, L = 60, 1560, 512
    g = torch.Generator().manual_seed(4321)
    video = torch.randn(frames * tokens, cfg.hidden, generator=g).bfloat16()
    text = torch.randn(L, cfg.hidden, generator=g).bfloat16()
    temb = torch.randn(cfg.hidden, generator=g)
    x = torch.cat([text, video])
    sample = [0, 29, 59]
    for i, block in enumerate(stack.blocks):
        out = block(x.to(cuda), temb.to(cuda), frames, tokens, text_rows=L)
        torch.cuda.synchronize()
        assert bool(torch.isfinite(out).all())
        w = _weights(block)
        w["o_b_softmax"] = block.o.bias.float().cpu()
        ref = oblock.block_reference(x, temb, w, frames, tokens, cfg, _reference_alpha(block),
                                     text_rows=L, out_frames=sample)
        got = _rows(out.cpu(), sample, tokens, L)
        err = _rel(got.float(), ref)
        assert err < 1e-2, (i, err)
        x = out.cpu()                                         # block 2 takes block 1's output
