"""One VDN-H3-style hybrid DiT block on the B200 kernels.

    x -> RMSNorm * (1 + scale_msa) + shift_msa -> [bf16 y1, MXFP8]      prenorm producer
      -> QKV (MXFP8 GEMM, N = 3 * hidden)
      -> gates from y1: softmax gate [T,H], beta [T,H], output-gate hidden [T,r]
         (one bf16 GEMM), linear gate [T,H*d] = sigmoid(up(hidden))
      -> frame mean of y1 -> alpha (FrameKDAAlpha)
      -> [Ulysses: sequence -> heads all-to-all]
      -> window softmax (+-radius frames) * softmax gate     cuDNN legs + vdn_window_merge
      -> VDA linear branch                                    vdn_vda_forward
      -> [Ulysses: heads -> sequence all-to-all]
      -> x1 = x + gate_msa * (to_out(softmax) + to_out_linear(VDA))   one dual-K MXFP8 GEMM
      -> RMSNorm * (1 + scale_mlp) + shift_mlp -> MXFP8 -> FFN up (MXFP8 GEMM)
      -> GELU -> MXFP8 -> FFN down, x2 = x1 + gate_mlp * ffn          fused GEMM epilogue

The pieces follow the reference: the pre-norm producer and gated residual of
src/models/ops/fused_block.py:43-51 / mxfp8_kernels.py:86-139, the hybrid
attention merge of src/models/hybrid_attention.py:178-255 (to_out + to_out_linear
on the video rows), the standard Ulysses forward of
src/inference/utils/ulysses.py:271-419, its branch-parallel forward (:421-598)
and the branch of src/models/linear_attention/branch.py.  The BASELINE block has
no RoPE / QK-norm and no text rows; the FFN is GELU (tanh form) rather than H3's
SwiGLU.  Weights are random (seeded), with a rank-32 LoRA merged into Q, K, V and
O before MXFP8 quantisation, as the reference merges before conversion.

Layouts beyond the BASELINE window (text rows packed first, anchor frames,
chunk-aligned windows, the text-seeded scans) take `_forward_general`: one GPU,
or Ulysses through the all-to-all exchange.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib
from .gates import gate_gemm
from .linear_attention import FrameKDAAlpha, OutputGate, frame_sums, window_bounds
from .mxfp8_kernels import launch_prenorm_quantize
from .mxfp8_quant import quantize_cpu, quantize_activation
from .window import window_softmax

__all__ = ["HybridBlock", "BlockConfig", "BlockGraph", "BlockPipeline"]


class BlockConfig:
    """Block geometry and the attention layout knobs of HybridAttention
    (src/models/hybrid_attention.py:45-80): `radius` / `chunk` (frame window, or
    K-frame chunk-aligned window when chunk > 0), `anchor_frames` ("none",
    "columns", "rows", "both"; "both" also drops frames 0 and F-1 from the linear
    branch) and `text_state` (seed both VDA scans with half the prompt state)."""

    def __init__(self, hidden=5120, heads=40, head_dim=128, ffn=13824, radius=1, lora_rank=32,
                 eps=1e-6, gelu="tanh", chunk=0, anchor_frames="none", text_state=False):
        self.hidden, self.heads, self.head_dim, self.ffn = hidden, heads, head_dim, ffn
        self.radius, self.lora_rank, self.eps, self.gelu = radius, lora_rank, eps, gelu
        if anchor_frames not in ("none", "columns", "rows", "both"):
            raise ValueError(f"anchor_frames={anchor_frames!r}")
        if chunk < 0 or radius < 0:
            raise ValueError("radius and chunk must be >= 0")
        self.chunk, self.anchor_frames, self.text_state = chunk, anchor_frames, bool(text_state)

    @property
    def plain_window(self) -> bool:
        """The BASELINE config-3 layout: a +-radius frame window, no anchors."""
        return self.chunk == 0 and self.anchor_frames == "none"


class _Packed:
    """MXFP8 weight (codes, swizzled scales) + optional bf16 bias, resident on device."""

    def __init__(self, w: torch.Tensor, bias: torch.Tensor | None, device):
        self.n, self.k = w.shape
        if w.is_cuda:  # weights drawn on the device: the device quantiser (same rule, bf16 input)
            q, s = quantize_activation(w.to(torch.bfloat16).contiguous(), check_finite=False)
        else:
            q, s = quantize_cpu(w.float())
        self.q, self.s = q.to(device), s.to(device)
        self.bias = None if bias is None else bias.to(torch.bfloat16).to(device)
        self.n_pad, self.k_pad = q.shape


class HybridBlock(nn.Module):
    """One hybrid block with random (seeded) weights.

    init="host" (default) draws every weight on the CPU and quantises with the
    host quantiser, so all Ulysses ranks and the CPU oracle see identical
    weights; init="device" draws the weights with a CUDA generator and quantises
    them on the device (bf16-rounded first): seconds instead of minutes for a
    40-block stack, for throughput runs that compare against no oracle.
    """

    def __init__(self, cfg: BlockConfig | None = None, *, seed=0, device="cuda", init="host"):
        super().__init__()
        cfg = cfg or BlockConfig()
        self.cfg = cfg
        hd, H, d = cfg.hidden, cfg.heads, cfg.head_dim
        if H * d != hd:
            raise ValueError("heads * head_dim must equal hidden")
        if hd % 128 or cfg.ffn % 128:
            raise ValueError("hidden and ffn must be multiples of 128 (MXFP8 epilogues)")
        if init not in ("host", "device"):
            raise ValueError("init must be 'host' or 'device'")
        dev = torch.device(device)
        gdev = dev if init == "device" else torch.device("cpu")
        g = torch.Generator(device=gdev).manual_seed(seed)

        def rnd(*shape, std=0.02):
            return torch.randn(*shape, generator=g, device=gdev) * std

        def lora(w):
            r = cfg.lora_rank
            a = torch.randn(r, w.shape[1], generator=g, device=gdev) * (1.0 / r) ** 0.5
            b = torch.randn(w.shape[0], r, generator=g, device=gdev) * 0.02
            return w + b @ a

        wq, wk, wv = (lora(rnd(hd, hd)) for _ in range(3))
        self.qkv = _Packed(torch.cat([wq, wk, wv]), rnd(3 * hd), dev)
        self.o = _Packed(lora(rnd(hd, hd)), rnd(hd), dev)
        self.ol = _Packed(rnd(hd, hd), rnd(hd), dev)
        self.up = _Packed(rnd(cfg.ffn, hd), rnd(cfg.ffn), dev)
        self.down = _Packed(rnd(hd, cfg.ffn), rnd(hd), dev)
        self.o_bias = (self.o.bias.float() + self.ol.bias.float()).to(torch.bfloat16)
        # bf16 small projections (the reference keeps these unquantised).  Their
        # default initialisers draw from the global generator: seed it here so
        # that every Ulysses rank builds the same weights.
        with torch.random.fork_rng(devices=[dev] if init == "device" else []):
            torch.manual_seed(seed + 0x5EED)
            mk = dict(device=dev) if init == "device" else {}
            self.adaln = nn.Linear(hd, 6 * hd, **mk).to(dev, torch.bfloat16)
            self.softmax_gate = nn.Linear(hd, H).to(dev, torch.bfloat16)
            nn.init.zeros_(self.softmax_gate.weight)
            nn.init.constant_(self.softmax_gate.bias, math.log(0.99 / 0.01))
            self.beta_proj = nn.Linear(hd, H, bias=False).to(dev, torch.bfloat16)
            self.output_gate = OutputGate(hd, H, d, bottleneck=d, init="random").to(dev, torch.bfloat16)
            self.alpha = FrameKDAAlpha(hd, H, d).to(dev)
        self.norm1 = torch.ones(hd, device=dev)
        self.norm2 = torch.ones(hd, device=dev)
        self.vda_norm = torch.ones(d, device=dev)
        self.eval()
        self._status = torch.zeros(1, dtype=torch.int32, device=dev)

    # ---------------------------------------------------------------- helpers
    def _gemm(self, a_q, a_s, w: _Packed, rows, out, *, second=None, bias=None, resid=None, gate=None):
        m_pad = a_q.shape[0]
        aq2 = as2 = wq2 = ws2 = None
        k2 = 0
        if second is not None:
            (aq2, as2), w2 = second
            wq2, ws2, k2 = w2.q, w2.s, w2.k_pad
        _lib.call("vdn_mxfp8_gemm_fused", _lib.ptr(a_q), _lib.ptr(a_s), _lib.ptr(w.q), _lib.ptr(w.s),
                  w.k_pad, _lib.ptr(aq2), _lib.ptr(as2), _lib.ptr(wq2), _lib.ptr(ws2), k2,
                  _lib.ptr(bias), m_pad, w.n, w.n_pad, rows, _lib.ptr(out), out.stride(0),
                  _lib.ptr(resid), resid.stride(0) if resid is not None else 0, _lib.ptr(gate),
                  _lib.ptr(self._status), _lib.stream_of(out.device))
        return out

    def _gate_projections(self, y1, out=None):
        """[rows, 2H + r]: sigmoid(softmax gate) | sigmoid(beta) | output-gate hidden, from
        ONE bf16 GEMM over y1 (the three projections share their input; their weights
        are concatenated once and re-concatenated only when a weight changes)."""
        og = self.output_gate
        ws = (self.softmax_gate.weight, self.beta_proj.weight, og.down.weight)
        key = tuple((w.data_ptr(), w._version) for w in ws) + (self.softmax_gate.bias._version,)
        if getattr(self, "_gate_key", None) != key:
            H = self.cfg.heads
            self._gate_w = torch.cat(ws, dim=0).contiguous()
            bias = torch.zeros(self._gate_w.shape[0], dtype=self._gate_w.dtype, device=self._gate_w.device)
            bias[:H] = self.softmax_gate.bias
            self._gate_b = bias
            self._gate_key = key
        H = self.cfg.heads
        return gate_gemm(y1, self._gate_w, self._gate_b, n_sig=2 * H, out=out)

    def _linear_gate(self, hidden, cols=slice(None)):
        """The VDA output gate sigmoid(up(hidden)) for output columns `cols` (a head
        range of H*d): [rows, len(cols)] bf16, on the tcgen05 gate GEMM."""
        og = self.output_gate
        w, b = og.up.weight[cols], og.up.bias[cols]
        return gate_gemm(hidden, w, b, n_sig=w.shape[0])

    def _side(self, device):
        """The branch-overlap stream of this device (the reference's vda_on_side_stream,
        src/inference/utils/vda_overlap.py:7-44): the VDA branch runs there while the
        window softmax runs on the caller's stream."""
        st = getattr(self, "_side_streams", None)
        if st is None:
            st = self._side_streams = {}
        if device.index not in st:
            st[device.index] = torch.cuda.Stream(device)
        return st[device.index]

    def _vda_side(self, fn, device):
        """Run fn() on the side stream after the caller's pending work; returns
        (result, join) where join() makes the caller's stream wait for it."""
        main = torch.cuda.current_stream(device)
        side = self._side(device)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            out = fn()
        done = torch.cuda.Event()
        done.record(side)

        def join():
            main.wait_event(done)
            for t in (out if isinstance(out, tuple) else (out,)):
                if isinstance(t, torch.Tensor):
                    t.record_stream(main)
            return out
        return join

    # ---------------------------------------------------------------- forward
    @torch.no_grad()
    def forward(self, x, temb, frames, tokens, runtime=None, text_rows=0):
        """x: this rank's rows [T_local, hidden] bf16 (all T rows when runtime is None).

        text_rows > 0: x is the packed sequence [text_rows + frames * tokens, hidden] (or
        this rank's rows of it), prompt rows first as global rows: dense softmax in both
        directions, no linear-branch output, and (cfg.text_state) the prompt seeds both
        VDA scans.  With such a layout (or anchors / chunk windows) a runtime must use
        exchange_mode "alltoall".
        """
        cfg = self.cfg
        hd, H, d = cfg.hidden, cfg.heads, cfg.head_dim
        T = frames * tokens
        rows = x.shape[0]
        dev = x.device
        general = text_rows > 0 or not cfg.plain_window
        if general:
            if runtime is not None and runtime.world_size > 1:
                if runtime.exchange_mode != "alltoall" or runtime.branch_parallel:
                    raise ValueError("text rows, anchor frames and chunk windows shard through the "
                                     "standard all-to-all exchange (exchange_mode='alltoall')")
                if runtime.sequence_length != text_rows + T or rows != runtime.local_end - runtime.local_start:
                    raise ValueError("configure the runtime for text_rows + frames * tokens rows")
                return self._forward_general(x, temb, frames, tokens, text_rows, runtime)
            if rows != text_rows + T:
                raise ValueError("x must hold text_rows + frames * tokens rows")
            return self._forward_general(x, temb, frames, tokens, text_rows)
        ev = runtime.profile_start() if runtime is not None else None
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = self._adaln(temb)
        idx = self._row_index(rows, dev)
        y1, q1, s1, _ = launch_prenorm_quantize(x, self.norm1, cfg.eps, scale_msa.view(1, hd),
                                                shift_msa.view(1, hd), idx, write_bf16=True)
        if runtime is not None:
            runtime.profile_end("adaln_prenorm", ev)
        if runtime is not None and runtime.world_size > 1 and runtime.branch_parallel:
            qkv = torch.empty(rows, 3 * hd, device=dev, dtype=torch.bfloat16)
            self._gemm(q1, s1, self.qkv, rows, qkv, bias=self.qkv.bias)
            first, second = self._attention_branch_parallel(qkv, self._gate_projections(y1), y1, frames,
                                                            tokens, runtime)
        elif runtime is not None and runtime.world_size > 1 and runtime.exchange_mode == "peer":
            first, second = self._attention_peer(y1, q1, s1, frames, tokens, runtime)
            ev = runtime.profile_start()
            x1 = torch.empty_like(x)
            self._gemm(first[0], first[1], self.o, rows, x1, second=(second, self.ol),
                       bias=self.o_bias, resid=x, gate=gate_msa.contiguous())
            runtime.profile_end("out_gemm", ev)
            ev = runtime.profile_start()
            x2 = self._ffn(x1, shift_mlp, scale_mlp, gate_mlp, idx)
            runtime.profile_end("ffn", ev)
            return x2
        else:
            qkv = torch.empty(rows, 3 * hd, device=dev, dtype=torch.bfloat16)
            self._gemm(q1, s1, self.qkv, rows, qkv, bias=self.qkv.bias)
            g3 = self._gate_projections(y1)                               # [rows, 2H + r]
            sgate, beta = g3[:, :H], g3[:, H:2 * H]                       # [rows, H] each
            og = self.output_gate
            lgate = self._linear_gate(g3[:, 2 * H:])                      # [rows, H*d]
            if runtime is None:
                frame_mean = frame_sums(y1, [f * tokens for f in range(frames + 1)], tokens)
                first, second = self._attention(qkv, sgate, beta, lgate, frame_mean, frames, tokens,
                                                heads=slice(0, H))
            else:
                first, second = self._attention_ulysses(qkv, sgate, beta, lgate, y1, frames, tokens,
                                                        runtime)
        x1 = torch.empty_like(x)
        self._gemm(first[0], first[1], self.o, rows, x1, second=(second, self.ol),
                   bias=self.o_bias, resid=x, gate=gate_msa.contiguous())
        return self._ffn(x1, shift_mlp, scale_mlp, gate_mlp, idx)

    def _row_index(self, rows, dev):
        """The AdaLN row -> modulation-row map (all rows use row 0: one timestep per
        call), cached per row count so a forward launches no fill for it."""
        cache = self.__dict__.setdefault("_row_index_cache", {})
        idx = cache.get((rows, dev))
        if idx is None:
            idx = cache[(rows, dev)] = torch.zeros(rows, dtype=torch.int64, device=dev)
        return idx

    def _adaln(self, temb):
        hd = self.cfg.hidden
        return self.adaln(F.silu(temb.to(torch.bfloat16)).view(1, hd)).view(6, hd)

    def _ffn(self, x1, shift_mlp, scale_mlp, gate_mlp, idx):
        """x2 = x1 + gate_mlp * FFN(prenorm(x1)) (GELU-tanh and its MXFP8 quantise fused into
        the FFN-up epilogue)."""
        cfg = self.cfg
        hd, rows, dev = cfg.hidden, x1.shape[0], x1.device
        _, q2, s2, _ = launch_prenorm_quantize(x1, self.norm2, cfg.eps, scale_mlp.view(1, hd),
                                               shift_mlp.view(1, hd), idx, write_bf16=False)
        w = self.up
        q3 = torch.empty(q2.shape[0], w.n, device=dev, dtype=torch.uint8)
        s3 = torch.empty(q2.shape[0] * w.n // 32, device=dev, dtype=torch.uint8)
        if cfg.gelu != "tanh":
            raise ValueError("the fused FFN epilogue implements GELU (tanh)")
        _lib.call("vdn_mxfp8_gemm_act_quantize", _lib.ptr(q2), _lib.ptr(s2), _lib.ptr(w.q), _lib.ptr(w.s),
                  w.k_pad, _lib.ptr(w.bias), q2.shape[0], w.n, w.n_pad, rows, _lib.ACT_GELU_TANH,
                  _lib.ptr(q3), _lib.ptr(s3), _lib.ptr(self._status), _lib.stream_of(dev))
        x2 = torch.empty_like(x1)
        self._gemm(q3, s3, self.down, rows, x2, bias=self.down.bias, resid=x1, gate=gate_mlp.contiguous())
        return x2

    def _forward_general(self, x, temb, frames, tokens, L, runtime=None):
        """Block with text rows, anchor frames and / or chunk-aligned windows
        (hybrid_attention.py:178-255 with branch.py:256-402).

        The softmax covers every row (text rows dense, video rows their window plus
        the anchors); the VDA branch covers the video rows it owns (all of them, or
        frames 1..F-2 under anchor_frames == "both") and is skipped when every window
        spans the clip.  The output projection runs as two GEMMs: the text rows take
        to_out alone, the video rows to_out + to_out_linear in one dual-K accumulator.
        With a runtime (world_size > 1, the all-to-all exchange) x holds this rank's
        rows of the packed sequence [text | video] and attention runs on H / P heads
        of all rows between the two exchanges (ulysses.py:271-419).
        """
        cfg = self.cfg
        hd, H, d = cfg.hidden, cfg.heads, cfg.head_dim
        T = frames * tokens
        n = x.shape[0]
        dev = x.device
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = self._adaln(temb)
        idx = self._row_index(n, dev)
        y1, q1, s1, _ = launch_prenorm_quantize(x, self.norm1, cfg.eps, scale_msa.view(1, hd),
                                                shift_msa.view(1, hd), idx, write_bf16=True)
        qkv = torch.empty(n, 3 * hd, device=dev, dtype=torch.bfloat16)
        self._gemm(q1, s1, self.qkv, n, qkv, bias=self.qkv.bias)
        g3 = self._gate_projections(y1)
        og = self.output_gate
        if runtime is None:
            q = qkv[:, :hd].view(n, H, d)
            k = qkv[:, hd:2 * hd].view(n, H, d)
            v = qkv[:, 2 * hd:].view(n, H, d)
            lgate = self._linear_gate(g3[L:, 2 * H:]).view(T, H, d)
            frame_mean = frame_sums(y1[L:], [f * tokens for f in range(frames + 1)], tokens)
            att = torch.empty(n, H, d, device=dev, dtype=torch.bfloat16)
            lin_q = self._layout_branches(q, k, v, g3[:, :H], g3[:, H:2 * H], lgate, frame_mean, frames,
                                          tokens, L, slice(0, H), att, quantize_lin=True)
            att = att.view(n, hd)
            local_text = L

            def quant_att(a, b):
                return quantize_activation(att[a:b], check_finite=False)
        else:
            rt = runtime
            hl = H // rt.world_size
            N = L + T
            sums, work = rt.video_frame_mean_async(y1, frames, tokens, video_start=L)
            lgate = self._linear_gate(g3[:, 2 * H:])
            # Per head: q | k | v | linear gate | softmax gate | beta | pad (W = 4d + 8).
            W = 4 * d + 8
            pack = torch.empty(n, H, W, device=dev, dtype=torch.bfloat16)
            pack[:, :, 0:3 * d] = qkv.view(n, 3, H, d).permute(0, 2, 1, 3).reshape(n, H, 3 * d)
            pack[:, :, 3 * d:4 * d] = lgate.view(n, H, d)
            pack[:, :, 4 * d] = g3[:, :H]
            pack[:, :, 4 * d + 1] = g3[:, H:2 * H]
            recv = rt.sequence_to_heads(pack)                             # [N, H/P, W]
            work.wait()
            frame_mean = sums / tokens
            h0 = rt.rank * hl
            ret = torch.empty(N, hl, 2 * d, device=dev, dtype=torch.bfloat16)
            lin = self._layout_branches(recv[:, :, 0:d], recv[:, :, d:2 * d], recv[:, :, 2 * d:3 * d],
                                        recv[:, :, 4 * d], recv[:, :, 4 * d + 1], recv[L:, :, 3 * d:4 * d],
                                        frame_mean, frames, tokens, L, slice(h0, h0 + hl), ret[:, :, :d],
                                        quantize_lin=False)
            ret[:L, :, d:].zero_()
            if lin is None:
                ret[L:, :, d:].zero_()
            else:
                ret[L:, :, d:] = lin.view(T, hl, d)
            flat = rt.heads_to_sequence(ret).view(n, H * 2 * d)           # [rows, H * 2d]
            local_text = max(0, min(L - rt.local_start, n))
            lin_q = None
            if lin is not None and n > local_text:
                lin_q = self._quantize_grouped(flat[local_text:], d, n - local_text)

            def quant_att(a, b):
                return self._quantize_grouped(flat[a:b], 0, b - a)
        x1 = self._project_out(x, quant_att, lin_q, local_text, gate_msa.contiguous())
        return self._ffn(x1, shift_mlp, scale_mlp, gate_mlp, idx)

    def _layout_branches(self, q, k, v, sgate, beta, lgate, frame_mean, frames, tokens, L, heads, att_out,
                         *, quantize_lin):
        """Window softmax over all [L + F*S, h, d] rows into att_out; the VDA branch over the
        video rows (lgate [F*S, h, d]) on the side stream.  Returns the VDA output (bf16
        [F*S, h*d], or its MXFP8 when quantize_lin), or None when every window spans the clip."""
        from .linear_attention import vda_forward, vda_text_seed
        cfg = self.cfg
        h, d = q.shape[1], q.shape[2]
        T = frames * tokens
        dev = q.device
        bounds = window_bounds(frames, cfg.radius, cfg.chunk)
        linear_active = not all(lo <= 0 and hi >= frames - 1 for lo, hi in bounds)

        def branch():  # VDA over the video rows, on the side stream
            alpha = self.alpha.forward_native(frame_mean, heads=heads)
            seed = vda_text_seed(k[:L], v[:L], beta[:L], 0.5) if cfg.text_state and L else None
            qv, kv, vv, bv = q[L:], k[L:], v[L:], beta[L:]
            if cfg.anchor_frames != "both":
                lin = vda_forward(qv, kv, vv, bv, lgate, alpha, bounds, frames, tokens, self.vda_norm,
                                  seed=seed)
            else:  # frames 0 and F-1 are exact softmax: dropped from the branch, rows zero
                lin = torch.zeros(T, h * d, device=dev, dtype=torch.bfloat16)
                if frames > 2:
                    inner = slice(tokens, (frames - 1) * tokens)
                    lin[inner] = vda_forward(qv[inner], kv[inner], vv[inner], bv[inner], lgate[inner],
                                             alpha[1:-1].contiguous(),
                                             [(lo - 1, hi - 1) for lo, hi in bounds[1:frames - 1]],
                                             frames - 2, tokens, self.vda_norm, seed=seed)
            return quantize_activation(lin, check_finite=False) if quantize_lin else lin

        join = self._vda_side(branch, dev) if linear_active else None
        window_softmax(q, k, v, sgate, frames, tokens, cfg.radius, out=att_out,
                       bounds=bounds, text_rows=L, anchor_frames=cfg.anchor_frames)
        return join() if join is not None else None

    def _project_out(self, x, quant_att, lin_q, text_rows, gate_msa):
        """x1 = x + gate_msa * (to_out(softmax) [+ to_out_linear(VDA) on the video rows]):
        rows [0, text_rows) take to_out alone (hybrid_attention.py:250-255)."""
        n = x.shape[0]
        x1 = torch.empty_like(x)
        if text_rows:
            aq, as_ = quant_att(0, text_rows)
            self._gemm(aq, as_, self.o, text_rows, x1[:text_rows], bias=self.o.bias, resid=x[:text_rows],
                       gate=gate_msa)
        if n > text_rows:
            aq, as_ = quant_att(text_rows, n)
            if lin_q is None:
                self._gemm(aq, as_, self.o, n - text_rows, x1[text_rows:], bias=self.o.bias,
                           resid=x[text_rows:], gate=gate_msa)
            else:
                self._gemm(aq, as_, self.o, n - text_rows, x1[text_rows:], second=(lin_q, self.ol),
                           bias=self.o_bias, resid=x[text_rows:], gate=gate_msa)
        return x1

    def _attention(self, qkv, sgate, beta, lgate, frame_mean, frames, tokens, heads):
        """Single-GPU attention: returns ((codes, scales) softmax, (codes, scales) VDA)."""
        from .linear_attention import vda_forward
        cfg = self.cfg
        hd, H, d = cfg.hidden, cfg.heads, cfg.head_dim
        T = frames * tokens
        q = qkv[:, :hd].view(T, H, d)
        k = qkv[:, hd:2 * hd].view(T, H, d)
        v = qkv[:, 2 * hd:].view(T, H, d)
        bounds = window_bounds(frames, cfg.radius)

        def branch():
            alpha = self.alpha.forward_native(frame_mean, heads=heads)
            lin = vda_forward(q, k, v, beta, lgate.view(T, H, d), alpha, bounds, frames, tokens,
                              self.vda_norm)
            return quantize_activation(lin, check_finite=False)

        join = self._vda_side(branch, qkv.device)
        att = window_softmax(q, k, v, sgate, frames, tokens, cfg.radius, quantize=True)
        return att, join()

    def _attention_ulysses(self, qkv, sgate, beta, lgate, y1, frames, tokens, rt):
        """Head-sharded attention between the two Ulysses exchanges."""
        from .linear_attention import vda_forward
        cfg = self.cfg
        hd, H, d = cfg.hidden, cfg.heads, cfg.head_dim
        T = frames * tokens
        rows = qkv.shape[0]
        P = rt.world_size
        hl = H // P
        sums, work = rt.video_frame_mean_async(y1, frames, tokens)
        # Pack per head: q | k | v | linear gate | softmax gate | beta | pad -> W = 4d + 8.
        W = 4 * d + 8
        pack = torch.empty(rows, H, W, device=qkv.device, dtype=torch.bfloat16)
        pack[:, :, 0:3 * d] = qkv.view(rows, 3, H, d).permute(0, 2, 1, 3).reshape(rows, H, 3 * d)
        pack[:, :, 3 * d:4 * d] = lgate.view(rows, H, d)
        pack[:, :, 4 * d] = sgate
        pack[:, :, 4 * d + 1] = beta
        recv = rt.sequence_to_heads(pack)                                 # [T, H/P, W]
        work.wait()
        frame_mean = sums / tokens
        first = rt.rank * hl
        heads = slice(first, first + hl)
        q, k, v = recv[:, :, 0:d], recv[:, :, d:2 * d], recv[:, :, 2 * d:3 * d]
        ret = torch.empty(T, hl, 2 * d, device=qkv.device, dtype=torch.bfloat16)
        window_softmax(q, k, v, recv[:, :, 4 * d], frames, tokens, cfg.radius, out=ret[:, :, :d])
        alpha = self.alpha.forward_native(frame_mean, heads=heads)
        bounds = window_bounds(frames, cfg.radius)
        lin = vda_forward(q, k, v, recv[:, :, 4 * d + 1], recv[:, :, 3 * d:4 * d], alpha, bounds,
                          frames, tokens, self.vda_norm)
        ret[:, :, d:] = lin.view(T, hl, d)
        back = rt.heads_to_sequence(ret)                                  # [rows, H, 2d]
        flat = back.view(rows, H * 2 * d)
        att = self._quantize_grouped(flat, 0, rows)
        lq = self._quantize_grouped(flat, d, rows)
        return att, lq

    def _attention_branch_parallel(self, qkv, g3, y1, frames, tokens, rt):
        """Branch-parallel attention (src/inference/utils/ulysses.py:421-598): the softmax
        ranks run the gated window softmax and the linear ranks the VDA branch, each
        for its own contiguous share of ALL heads.

        QKV is projected once by every sequence owner; one uneven all-to-all per
        branch (two communicators) sends q | k | v | softmax gate to the softmax
        ranks and q | k | v | beta plus the output gate's low-rank hidden to the
        linear ranks, which apply the gate's `up` half to their own heads only.  One
        reverse all-to-all returns both branches' heads to the sequence owner, where
        each is quantised on its own (its own block scales) into the dual-K output
        GEMM.
        """
        from .linear_attention import vda_forward
        cfg = self.cfg
        hd, H, d = cfg.hidden, cfg.heads, cfg.head_dim
        T = frames * tokens
        rows = qkv.shape[0]
        sums, work = rt.video_frame_mean_async(y1, frames, tokens)
        q = qkv[:, :hd].view(rows, H, d)
        k = qkv[:, hd:2 * hd].view(rows, H, d)
        v = qkv[:, 2 * hd:].view(rows, H, d)
        packed, shared, pending = rt.dispatch_fields_to_branches_overlapped(
            q, k, v, g3[:, :H], q, k, g3[:, H:2 * H], g3[:, 2 * H:])
        work.wait()
        frame_mean = sums / tokens
        hb, h0 = rt.branch_heads, rt.branch_first_head
        # The wire rows are 3d + 1 wide; the kernels want 16-byte aligned operands.
        fields = packed[:, :, :3 * d].contiguous()                        # [T, hb, 3d]
        scalar = packed[:, :, 3 * d].contiguous()                         # [T, hb]
        qh, kh, vh = fields[:, :, :d], fields[:, :, d:2 * d], fields[:, :, 2 * d:]
        if rt.branch_kind == "softmax":
            out = torch.empty(T, hb, d, device=qkv.device, dtype=torch.bfloat16)
            window_softmax(qh, kh, vh, scalar, frames, tokens, cfg.radius, out=out)
        else:
            og = self.output_gate
            cols = slice(h0 * d, (h0 + hb) * d)
            lgate = self._linear_gate(shared, cols)
            alpha = self.alpha.forward_native(frame_mean, heads=slice(h0, h0 + hb))
            out = vda_forward(qh, kh, vh, scalar, lgate.view(T, hb, d), alpha,
                              window_bounds(frames, cfg.radius), frames, tokens,
                              self.vda_norm).view(T, hb, d)
        pending[0].wait()
        del pending
        softmax_local, linear_local = rt.branches_to_sequence(out)        # [rows, H, d] each
        att = quantize_activation(softmax_local.view(rows, hd), check_finite=False)
        lq = quantize_activation(linear_local.view(rows, hd), check_finite=False)
        return att, lq

    def _attention_peer(self, y1, q1, s1, frames, tokens, rt):
        """Head-sharded attention with the exchange done by the producers (peer memory).

        The QKV GEMM stores every head's slice into its owner's receive buffer;
        the softmax / VDA outputs return as MXFP8 through the scatter quantiser.
        The small per-token gate inputs (softmax gate, beta, the output gate's
        low-rank hidden) and the per-rank frame sums for alpha are copied into
        every rank by the copy engines while the QKV GEMM runs.
        """
        from .linear_attention import vda_forward
        cfg = self.cfg
        hd, H, d = cfg.hidden, cfg.heads, cfg.head_dim
        T = frames * tokens
        og = self.output_gate
        r = og.down.weight.shape[0]
        ex = rt.exchange(H, d, frames, 2 * H + r)
        hl, h0 = ex.hl, ex.head0
        # Side inputs into this rank's slot of every rank's buffers (copy engines).
        ev = rt.profile_start()
        rt.local_frame_sums(y1, frames, tokens, out=ex.sums()[rt.rank])
        ex.publish_sums()
        self._gate_projections(y1, out=ex.local_rows())                  # [rows, 2H + r]
        ex.publish_rows()
        rt.profile_end("gates_and_side_rows", ev)
        ev = rt.profile_start()
        w = self.qkv
        _lib.call("vdn_mxfp8_gemm_scatter", _lib.ptr(q1), _lib.ptr(s1), _lib.ptr(w.q), _lib.ptr(w.s),
                  w.k_pad, _lib.ptr(w.bias), q1.shape[0], w.n, w.n_pad, y1.shape[0],
                  _lib.ptr(ex.chunk_dst), ex.dst_ld, rt.local_start, _lib.ptr(self._status),
                  _lib.stream_of(y1.device))
        rt.profile_end("qkv_gemm_scatter", ev)
        ev = rt.profile_start()
        ex.fence()
        rt.profile_end("fence_heads", ev)
        gathered = ex.rows()                                              # [T, 2H + r]
        frame_mean = ex.sums().sum(0) / tokens                            # fixed rank order
        recv = ex.qkv()                                                   # [T, hl, 3d]
        q, k, v = recv[:, :, 0:d], recv[:, :, d:2 * d], recv[:, :, 2 * d:3 * d]
        cols = slice(h0 * d, (h0 + hl) * d)
        lgate = self._linear_gate(gathered[:, 2 * H:], cols)
        bounds = window_bounds(frames, cfg.radius)

        def branch():  # VDA and its return scatter, on the side stream
            ev = rt.profile_start()
            alpha = self.alpha.forward_native(frame_mean, heads=slice(h0, h0 + hl))
            lin = vda_forward(q, k, v, gathered[:, H + h0:H + h0 + hl], lgate.view(T, hl, d), alpha,
                              bounds, frames, tokens, self.vda_norm)
            rt.profile_end("vda_branch", ev)
            ev = rt.profile_start()
            ex.scatter_quantize(lin.view(T, hl, d), ex.lin_dst)
            rt.profile_end("vda_quantize_scatter", ev)
            return lin

        join = self._vda_side(branch, y1.device)
        ev = rt.profile_start()
        att = torch.empty(T, hl, d, device=y1.device, dtype=torch.bfloat16)
        window_softmax(q, k, v, gathered[:, h0:h0 + hl], frames, tokens, cfg.radius, out=att)
        rt.profile_end("window_softmax", ev)
        ev = rt.profile_start()
        ex.scatter_quantize(att, ex.att_dst)
        rt.profile_end("softmax_quantize_scatter", ev)
        join()
        ev = rt.profile_start()
        ex.fence()
        rt.profile_end("fence_rows", ev)
        return ex.operands()

    def _quantize_grouped(self, flat, offset, rows):
        cfg = self.cfg
        hd, d = cfg.hidden, cfg.head_dim
        rp = (rows + 127) // 128 * 128
        q = torch.empty(rp, hd, dtype=torch.uint8, device=flat.device)
        s = torch.empty(rp * hd // 32, dtype=torch.uint8, device=flat.device)
        src = flat[:, offset:]
        _lib.call("vdn_mxfp8_quantize_grouped", _lib.C.c_void_p(src.data_ptr()), rows, hd,
                  flat.stride(0), d, 2 * d, _lib.ptr(q), _lib.ptr(s), None,
                  _lib.stream_of(flat.device))
        return q, s


class BlockGraph:
    """One block forward captured as a CUDA graph: the launch-bound host work of
    the ~50 launches per forward is replayed by the driver in one call.

    Inputs and output are static tensors: copy new rows into `x` (and `temb`),
    call replay(), read `out`.  The eager forwards run first on a side stream
    create every lazily built resource (library state, cuDNN plans, the Ulysses
    peer exchange), which must not happen during capture.  Only the peer
    exchange runs under a graph at world_size > 1 (its fences take their epoch
    from a device counter, so replays stay in step across ranks).
    """

    def __init__(self, block: HybridBlock, x, temb, frames, tokens, runtime=None, warmup=2):
        if runtime is not None and runtime.world_size > 1 and (runtime.exchange_mode != "peer"
                                                               or runtime.branch_parallel):
            raise ValueError("CUDA-graph capture needs the standard peer exchange at world_size > 1")
        self.block, self.x, self.temb = block, x, temb
        self.frames, self.tokens, self.runtime = frames, tokens, runtime
        dev = x.device
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(max(1, warmup)):
                block(x, temb, frames, tokens, runtime)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = block(x, temb, frames, tokens, runtime)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out


class BlockPipeline:
    """Streams batches from pinned host memory through one block and back.

    Two CUDA graphs (each with its own static input / output) alternate, so the
    host-to-device copy of batch i+1 and the device-to-host copy of batch i-1
    run on the copy engines (two extra streams) while batch i computes.  Every
    batch still makes both of its copies; only their overlap with the compute
    of the neighbouring batches changes.
    """

    def __init__(self, block: HybridBlock, rows: int, temb, frames, tokens, runtime=None):
        dev = temb.device
        hidden = block.cfg.hidden
        self.graphs = [BlockGraph(block, torch.zeros(rows, hidden, device=dev, dtype=torch.bfloat16), temb,
                                  frames, tokens, runtime) for _ in range(2)]
        self.device = dev
        self.h2d = torch.cuda.Stream(dev)
        self.d2h = torch.cuda.Stream(dev)
        self.in_ready = [torch.cuda.Event() for _ in range(2)]
        self.computed = [torch.cuda.Event() for _ in range(2)]
        self.out_free = [torch.cuda.Event() for _ in range(2)]

    def run(self, host_inputs, host_outputs) -> None:
        """Enqueue len(host_inputs) batches (pinned [rows, hidden] bf16 host tensors;
        results into the matching host_outputs).  Returns once everything is queued on
        the caller's stream: synchronise before reading the outputs."""
        if len(host_inputs) != len(host_outputs):
            raise ValueError("one output buffer per input batch")
        main = torch.cuda.current_stream(self.device)
        self.h2d.wait_stream(main)
        self.d2h.wait_stream(main)
        for i, (src, dst) in enumerate(zip(host_inputs, host_outputs)):
            b = i & 1
            g = self.graphs[b]
            with torch.cuda.stream(self.h2d):
                if i >= 2:
                    self.h2d.wait_event(self.computed[b])      # batch i-2 no longer reads g.x
                g.x.copy_(src, non_blocking=True)
                self.in_ready[b].record(self.h2d)
            main.wait_event(self.in_ready[b])
            if i >= 2:
                main.wait_event(self.out_free[b])              # batch i-2's result has left g.out
            g.replay()
            self.computed[b].record(main)
            with torch.cuda.stream(self.d2h):
                self.d2h.wait_event(self.computed[b])
                dst.copy_(g.out, non_blocking=True)
                self.out_free[b].record(self.d2h)
        main.wait_stream(self.d2h)
        main.wait_stream(self.h2d)
