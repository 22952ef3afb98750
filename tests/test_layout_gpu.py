"""GPU: the attention layouts beyond the BASELINE window -- global text rows packed
first, anchor frames, chunk-aligned windows, a window that spans the clip -- in the
window softmax and in the whole hybrid block, against the CPU references
(oracle.window, pinned to the reference's window_softmax_reference; oracle.block).
"""
import pytest
import torch

from oracle import block as oblock
from oracle import window as ow

from test_block_gpu import _reference_alpha, _rel, _weights

pytestmark = pytest.mark.gpu

WINDOW_CASES = [
    # text rows, frames, tokens, heads, head dim, radius, chunk, anchors
    (16, 5, 48, 2, 128, 1, 0, "both"),
    (7, 7, 40, 2, 64, 1, 2, "columns"),
    (0, 5, 64, 3, 128, 0, 0, "rows"),
    (5, 4, 33, 2, 128, 1, 0, "none"),
    (3, 9, 16, 1, 128, 2, 0, "both"),
    (0, 6, 32, 2, 128, 3, 0, "none"),
]


@pytest.mark.parametrize("L,f,s,h,d,radius,chunk,anchors", WINDOW_CASES)
@torch.no_grad()
def test_window_layouts_match_reference(cuda, L, f, s, h, d, radius, chunk, anchors):
    from vdn_b200.window import window_softmax
    g = torch.Generator().manual_seed(L * 100 + f + radius)
    n = L + f * s
    qkv = torch.randn(n, 3, h, d, generator=g).bfloat16()
    gate = torch.rand(n, h, generator=g).bfloat16()
    dq = qkv.to(cuda)
    out = torch.zeros(n, h, d, dtype=torch.bfloat16, device=cuda)
    bounds = ow.window_bounds(f, radius, chunk)
    codes = window_softmax(dq[:, 0], dq[:, 1], dq[:, 2], gate.to(cuda), f, s, radius, out=out,
                           quantize=True, bounds=bounds, text_rows=L, anchor_frames=anchors)
    torch.cuda.synchronize()
    ref = ow.window_attention(qkv[:, 0].float(), qkv[:, 1].float(), qkv[:, 2].float(), f, s, bounds,
                              d ** -0.5, text_rows=L, anchor_frames=anchors)
    ref = (ref.bfloat16().float() * gate.float()[..., None]).bfloat16().float()
    assert _rel(out.float(), ref) < 8e-3
    from vdn_b200.mxfp8_quant import quantize_activation
    q2, s2 = quantize_activation(out.view(n, h * d), check_finite=False)
    assert torch.equal(codes[0], q2) and torch.equal(codes[1], s2)


BLOCK_CASES = [
    # text rows, frames, tokens, radius, chunk, anchors, text_state
    (16, 5, 64, 1, 0, "both", True),
    (8, 6, 48, 1, 2, "columns", True),
    (0, 4, 64, 0, 0, "rows", False),
    (5, 3, 64, 3, 0, "none", False),          # the window spans the clip: no linear branch
    (0, 5, 40, 1, 0, "both", False),
]


@pytest.mark.parametrize("L,frames,tokens,radius,chunk,anchors,text_state", BLOCK_CASES)
@torch.no_grad()
def test_block_layouts_match_reference_composition(cuda, L, frames, tokens, radius, chunk, anchors,
                                                    text_state):
    from vdn_b200.block import BlockConfig, HybridBlock
    cfg = BlockConfig(hidden=256, heads=2, head_dim=128, ffn=512, radius=radius, lora_rank=8,
                      chunk=chunk, anchor_frames=anchors, text_state=text_state)
    block = HybridBlock(cfg, seed=1, device=cuda)
    torch.nn.init.normal_(block.softmax_gate.weight, std=0.05)
    g = torch.Generator().manual_seed(L * 1000 + frames * 10 + tokens)
    n = L + frames * tokens
    x = torch.randn(n, cfg.hidden, generator=g).bfloat16()
    temb = torch.randn(cfg.hidden, generator=g)
    out = block(x.to(cuda), temb.to(cuda), frames, tokens, text_rows=L)
    torch.cuda.synchronize()
    assert out.shape == (n, cfg.hidden) and bool(torch.isfinite(out).all())
    w = _weights(block)
    w["o_b_softmax"] = block.o.bias.float().cpu()
    ref = oblock.block_reference(x, temb, w, frames, tokens, cfg,
                                 _reference_alpha(block), text_rows=L)
    assert _rel(out.float(), ref) < 1e-2
    if L:
        assert _rel(out[:L].float(), ref[:L]) < 1e-2


@torch.no_grad()
def test_block_layouts_refuse_ulysses(cuda):
    from types import SimpleNamespace
    from vdn_b200.block import BlockConfig, HybridBlock
    cfg = BlockConfig(hidden=256, heads=2, head_dim=128, ffn=512, lora_rank=8, anchor_frames="both")
    block = HybridBlock(cfg, seed=1, device=cuda)
    x = torch.zeros(4 * 64, 256, dtype=torch.bfloat16, device=cuda)
    peer = SimpleNamespace(world_size=2, exchange_mode="peer", branch_parallel=False)
    with pytest.raises(ValueError):                       # layouts shard through the all-to-all only
        block(x, torch.zeros(256, device=cuda), 4, 64, peer)
    a2a = SimpleNamespace(world_size=2, exchange_mode="alltoall", branch_parallel=False,
                          sequence_length=4 * 64 + 8, local_start=0, local_end=132)
    with pytest.raises(ValueError):                       # runtime configured for another geometry
        block(x, torch.zeros(256, device=cuda), 4, 64, a2a)
    with pytest.raises(ValueError):
        block(x, torch.zeros(256, device=cuda), 4, 64, text_rows=3)
