"""GPU: the hybrid DiT block against a CPU fp32 composition of the reference pieces.

The reference composition (oracle/block.py) reproduces every MXFP8 quantisation
point bit-exactly and evaluates the rest in fp32 (window softmax by one SDPA per
frame, the VDA branch by the numpy oracle).  Tolerance on the block output:
relative L2 < 1e-2 (bf16 rounding points and rare one-code MXFP8 flips they
cause), and each sub-result is checked on its own first.
"""
import numpy as np
import pytest
import torch

from oracle import block as oblock
from oracle import mxfp8 as omx

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm())


def _deq(p):
    w = omx.dequantize(p.q.cpu().numpy(), p.s.cpu().numpy())[: p.n, : p.k]
    return torch.from_numpy(w).float()


def _weights(block):
    og = block.output_gate
    return dict(
        adaln_w=block.adaln.weight.float().cpu(), adaln_b=block.adaln.bias.float().cpu(),
        norm1=block.norm1.cpu(), norm2=block.norm2.cpu(),
        qkv=_deq(block.qkv), qkv_b=block.qkv.bias.float().cpu(),
        o=_deq(block.o), ol=_deq(block.ol), o_b=block.o_bias.float().cpu(),
        up=_deq(block.up), up_b=block.up.bias.float().cpu(),
        down=_deq(block.down), down_b=block.down.bias.float().cpu(),
        sg_w=block.softmax_gate.weight.float().cpu(), sg_b=block.softmax_gate.bias.float().cpu(),
        beta_w=block.beta_proj.weight.float().cpu(),
        og_down=og.down.weight.float().cpu(), og_up=og.up.weight.float().cpu(),
        og_b=og.up.bias.float().cpu())


def _small_block(cuda, seed=0):
    from vdn_b200.block import BlockConfig, HybridBlock
    cfg = BlockConfig(hidden=256, heads=2, head_dim=128, ffn=512, radius=1, lora_rank=8)
    block = HybridBlock(cfg, seed=seed, device=cuda)
    # Give the softmax gate live weights so the test exercises it.
    torch.nn.init.normal_(block.softmax_gate.weight, std=0.05)
    return cfg, block


@pytest.mark.parametrize("frames,tokens", [(4, 64), (3, 100)])
@torch.no_grad()
def test_block_matches_reference_composition(cuda, frames, tokens):
    cfg, block = _small_block(cuda)
    g = torch.Generator().manual_seed(frames * 1000 + tokens)
    T = frames * tokens
    x = torch.randn(T, cfg.hidden, generator=g).bfloat16()
    temb = torch.randn(cfg.hidden, generator=g)
    out = block(x.to(cuda), temb.to(cuda), frames, tokens)
    torch.cuda.synchronize()
    assert out.shape == (T, cfg.hidden) and out.dtype == torch.bfloat16
    assert bool(torch.isfinite(out).all())
    ref = oblock.block_reference(x, temb, _weights(block), frames, tokens, cfg, _reference_alpha(block))
    err = _rel(out.float(), ref)
    assert err < 1e-2, err


@torch.no_grad()
def test_window_softmax_matches_exact_window(cuda):
    from vdn_b200.window import window_softmax
    g = torch.Generator().manual_seed(5)
    frames, tokens, H, d = 5, 48, 2, 128
    T = frames * tokens
    q, k, v = (torch.randn(T, H, d, generator=g).bfloat16() for _ in range(3))
    gate = torch.rand(T, H, generator=g).bfloat16()
    out = torch.zeros(T, H, d, dtype=torch.bfloat16, device=cuda)
    codes = window_softmax(q.to(cuda), k.to(cuda), v.to(cuda), gate.to(cuda), frames, tokens, 1,
                           out=out, quantize=True)
    ref = oblock.window_attention(q.float(), k.float(), v.float(), frames, tokens, 1, d ** -0.5)
    ref = (ref.bfloat16().float() * gate.float()[..., None])
    assert _rel(out.float(), ref) < 5e-3
    # The MXFP8 output is exactly the quantisation of the bf16 output.
    rq, rs = omx.quantize(out.float().cpu().numpy().reshape(T, H * d))
    assert np.array_equal(codes[0].cpu().numpy(), rq) and np.array_equal(codes[1].cpu().numpy(), rs)


@pytest.mark.parametrize("m", [300, 500])   # 500 rows pad to 512: the CTA-pair kernel
@torch.no_grad()
def test_fused_gemm_dual_k_and_gated_residual(cuda, m):
    from vdn_b200 import _lib
    from vdn_b200.mxfp8_quant import quantize_activation
    g = torch.Generator(device=cuda).manual_seed(9)
    n, k1, k2 = 384, 256, 512
    x1 = torch.randn(m, k1, device=cuda, generator=g).bfloat16()
    x2 = torch.randn(m, k2, device=cuda, generator=g).bfloat16()
    w1 = (torch.randn(n, k1, device=cuda, generator=g) * 0.05).bfloat16()
    w2 = (torch.randn(n, k2, device=cuda, generator=g) * 0.05).bfloat16()
    (a1, s1), (a2, s2) = quantize_activation(x1), quantize_activation(x2)
    (b1, t1), (b2, t2) = quantize_activation(w1), quantize_activation(w2)
    bias = torch.randn(n, device=cuda, generator=g).bfloat16()
    resid = torch.randn(m, n, device=cuda, generator=g).bfloat16()
    gate = torch.rand(n, device=cuda, generator=g).bfloat16()
    y = torch.empty(m, n, device=cuda, dtype=torch.bfloat16)
    _lib.call("vdn_mxfp8_gemm_fused", _lib.ptr(a1), _lib.ptr(s1), _lib.ptr(b1), _lib.ptr(t1), k1,
              _lib.ptr(a2), _lib.ptr(s2), _lib.ptr(b2), _lib.ptr(t2), k2, _lib.ptr(bias), a1.shape[0],
              n, b1.shape[0], m, _lib.ptr(y), n, _lib.ptr(resid), n, _lib.ptr(gate), None,
              _lib.stream_of(cuda))
    torch.cuda.synchronize()
    deq = lambda q, s: torch.from_numpy(omx.dequantize(q.cpu().numpy(), s.cpu().numpy()))
    acc = deq(a1, s1)[:m, :k1] @ deq(b1, t1)[:n, :k1].T + deq(a2, s2)[:m, :k2] @ deq(b2, t2)[:n, :k2].T
    r = (acc.float().bfloat16().float() + bias.float().cpu()).bfloat16().float()
    want = (resid.float().cpu() + (gate.float().cpu() * r).bfloat16().float()).bfloat16()
    torch.testing.assert_close(y.cpu(), want, rtol=.01, atol=.02)


@torch.no_grad()
def test_block_graph_replay_matches_eager(cuda):
    """BlockGraph: replays of the captured forward equal eager forwards, for
    new inputs copied into the static buffer."""
    from vdn_b200.block import BlockGraph
    cfg, block = _small_block(cuda, seed=2)
    frames, tokens = 4, 64
    g = torch.Generator().manual_seed(77)
    xs = [torch.randn(frames * tokens, cfg.hidden, generator=g).bfloat16().to(cuda) for _ in range(2)]
    temb = torch.randn(cfg.hidden, generator=g).to(cuda)
    want = [block(x, temb, frames, tokens).clone() for x in xs]
    static = xs[0].clone()
    graph = BlockGraph(block, static, temb, frames, tokens)
    for x, w in zip(xs, want):
        static.copy_(x)
        out = graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, w)


def _reference_alpha(block):
    """Alpha from the block's own FrameKDAAlpha weights through the oracle's restatement
    (pinned to the reference's FrameKDAAlpha by tests/golden/alpha_golden.npz), so the
    block test does not take alpha from the module under test."""
    a = block.alpha
    w = [t.detach().float().cpu().numpy() for t in (a.down.weight, a.up.weight, a.dt_bias, a.A_log)]
    return oblock.alpha_fn(*w, a.num_heads, a.head_dim)


@pytest.mark.parametrize("case", ["small", "d128"])
@pytest.mark.parametrize("heads", [None, (1, 3)])
@torch.no_grad()
def test_frame_alpha_native_matches_reference_fixture(cuda, alpha_golden, case, heads):
    """vdn_frame_alpha (FrameKDAAlpha.forward_native) against the alpha the reference's
    FrameKDAAlpha produced from the same weights and frame means (layers.py:36-69)."""
    from vdn_b200.linear_attention import FrameKDAAlpha
    g = alpha_golden
    hidden, nh, d = (int(x) for x in g[case + "_geometry"])
    mod = FrameKDAAlpha(hidden, nh, d)
    mod.down.weight.copy_(torch.from_numpy(g[case + "_down"]))
    mod.up.weight.copy_(torch.from_numpy(g[case + "_up"]))
    mod.A_log.copy_(torch.from_numpy(g[case + "_a_log"]))
    mod.dt_bias.copy_(torch.from_numpy(g[case + "_dt_bias"]))
    mod = mod.to(cuda)
    fm = torch.from_numpy(g[case + "_frame_mean"]).to(cuda)
    sl = None if heads is None else slice(*heads)
    want = torch.from_numpy(g[case + ("_alpha" if heads is None else "_alpha_heads13")])
    got = mod.forward_native(fm, heads=sl).cpu()
    torch.testing.assert_close(got, want, rtol=2e-5, atol=1e-6)


@pytest.mark.parametrize("heads", [None, (2, 5)])
@torch.no_grad()
def test_frame_alpha_native_matches_module(cuda, heads):
    """vdn_frame_alpha == FrameKDAAlpha.forward (fp32, reference layers.py:36-69)."""
    from vdn_b200.linear_attention import FrameKDAAlpha
    torch.manual_seed(3)
    mod = FrameKDAAlpha(1024, 8, 128).to(cuda)
    fm = torch.randn(21, 1024, device=cuda)
    sl = None if heads is None else slice(*heads)
    torch.testing.assert_close(mod.forward_native(fm, heads=sl), mod(fm, heads=sl), rtol=2e-5, atol=1e-6)


@torch.no_grad()
def test_block_pipeline_matches_eager(cuda):
    """BlockPipeline: batches streamed from pinned host memory (copies overlapped with
    the neighbouring batches' compute) give the eager forward's outputs."""
    from vdn_b200.block import BlockPipeline
    cfg, block = _small_block(cuda, seed=4)
    frames, tokens = 4, 64
    T = frames * tokens
    g = torch.Generator().manual_seed(91)
    temb = torch.randn(cfg.hidden, generator=g).to(cuda)
    xs = [torch.randn(T, cfg.hidden, generator=g).bfloat16().pin_memory() for _ in range(5)]
    want = [block(x.to(cuda), temb, frames, tokens).cpu() for x in xs]
    outs = [torch.empty(T, cfg.hidden, dtype=torch.bfloat16).pin_memory() for _ in xs]
    pipe = BlockPipeline(block, T, temb, frames, tokens)
    pipe.run(xs, outs)
    torch.cuda.synchronize()
    for o, w in zip(outs, want):
        assert torch.equal(o, w)
