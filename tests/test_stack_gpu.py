"""GPU: the block stack and its denoise loop (BASELINE config 4's shape at toy size):
the stack equals its blocks applied in turn, the Euler loop equals its steps, and the
device-side weight initialisation gives a working block."""
import pytest
import torch

from test_block_gpu import _rel

pytestmark = pytest.mark.gpu


@torch.no_grad()
def test_stack_and_denoise_compose_blocks(cuda):
    from vdn_b200.block import BlockConfig
    from vdn_b200.stack import HybridStack, denoise
    cfg = BlockConfig(hidden=256, heads=2, head_dim=128, ffn=512, lora_rank=8, text_state=True)
    stack = HybridStack(cfg, depth=3, seed=2, device=cuda)
    frames, tokens, L = 4, 64, 16
    g = torch.Generator(device=cuda).manual_seed(9)
    video = torch.randn(frames * tokens, 256, device=cuda, generator=g).bfloat16()
    text = torch.randn(2, L, 256, device=cuda, generator=g).bfloat16()
    tembs = torch.randn(2, 256, device=cuda, generator=g)
    want = video.clone()
    for i in range(2):
        x = torch.cat([text[i], want])
        for blk in stack.blocks:
            x = blk(x, tembs[i], frames, tokens, text_rows=L)
        want = want + (-0.5) * x[L:]
    got = denoise(stack, video.clone(), text, tembs, frames, tokens)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(got).all())
    assert _rel(got.float(), want.float()) < 2e-2


@torch.no_grad()
def test_device_initialised_block_runs(cuda):
    from vdn_b200.block import BlockConfig, HybridBlock
    cfg = BlockConfig(hidden=256, heads=2, head_dim=128, ffn=512, lora_rank=8)
    a = HybridBlock(cfg, seed=5, device=cuda, init="device")
    b = HybridBlock(cfg, seed=5, device=cuda, init="device")
    assert torch.equal(a.qkv.q, b.qkv.q) and torch.equal(a.adaln.weight, b.adaln.weight)
    x = torch.randn(4 * 64, 256, device=cuda).bfloat16()
    temb = torch.randn(256, device=cuda)
    y = a(x, temb, 4, 64)
    torch.cuda.synchronize()
    assert bool(torch.isfinite(y).all()) and torch.equal(y, b(x, temb, 4, 64))
    with pytest.raises(ValueError):
        HybridBlock(cfg, device=cuda, init="meta")
