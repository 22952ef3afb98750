"""The VDA linear-attention branch on B200 kernels, behind the reference module API.

Mirrors ec-jt/vdn src/models/linear_attention/branch.py (BidirectionalLinearBranch,
its head-sharded forward signature, anchors and the text seed), layers.py
(FrameKDAAlpha), ops/rms_norm.py (RMSNorm), attention_gates.py (OutputGate) and
softmax_attention/window.py (window_bounds), plus the stage ops of paper_stack.py
(statistics, scans, gather) on the library's kernels.

The branch body is one C-ABI call, vdn_vda_forward: statistics, factors, both
scans, the boundary gather, the readout and the RMSNorm * gate epilogue run as
sm_100a kernels.  The small learnable pieces around it (beta and gate
projections when the caller does not supply them, the per-frame alpha island)
stay PyTorch modules with the reference's parameter names so checkpoints load
unchanged.  Inference only: forward requires torch.no_grad().  There is no CPU
or PyTorch fallback for the body.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from . import _lib
from .paper_factor import paper_delta_factors

__all__ = ["window_bounds", "RMSNorm", "OutputGate", "FrameKDAAlpha",
           "BidirectionalLinearBranch", "vda_statistics", "vda_scan", "vda_gather",
           "vda_forward", "vda_text_seed"]

BRIDGE_MODES = ("alpha", "none")
MAX_FRAMES = 1024


def window_bounds(num_frames, radius, chunk=0):
    """Per-frame inclusive window [lo, hi], unclamped (window.py:26-52)."""
    if chunk <= 0:
        return [(t - radius, t + radius) for t in range(num_frames)]
    return [(((t // chunk) - radius) * chunk, ((t // chunk) + radius + 1) * chunk - 1)
            for t in range(num_frames)]


class RMSNorm(nn.Module):
    """nn.RMSNorm-compatible parameters (weight [dim], eps) (ops/rms_norm.py:23-32)."""

    def __init__(self, dim, eps=1e-6):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        ms = torch.linalg.vector_norm(x, dim=-1, keepdim=True, dtype=torch.float32).pow(2) / x.shape[-1]
        return x * torch.rsqrt(ms + self.eps).to(x.dtype) * self.weight.to(x.dtype)


class OutputGate(nn.Module):
    """Sigmoid output gate, per head or per channel (attention_gates.py:13-55)."""

    def __init__(self, hidden_size, num_heads, head_dim=None, bottleneck=None,
                 init_value=0.9, init="constant"):
        super().__init__()
        self.num_heads, self.head_dim = num_heads, head_dim
        self.init_value = init_value
        out_features = num_heads * (head_dim or 1)
        self.down = None if bottleneck is None else nn.Linear(hidden_size, bottleneck, bias=False)
        self.up = nn.Linear(bottleneck or hidden_size, out_features, bias=True)
        if init == "constant":
            nn.init.zeros_(self.up.weight)
            nn.init.constant_(self.up.bias, math.log(init_value / (1.0 - init_value)))
        elif init != "random":
            raise ValueError(f"OutputGate init must be 'constant' or 'random', got {init!r}")

    def forward(self, x):
        gate = torch.sigmoid(self.up(x if self.down is None else self.down(x)))
        return gate.view(-1, self.num_heads, self.head_dim or 1)


def frame_sums(x, bounds, divisor=1.0, out=None):
    """Per-frame fp32 column sums of bf16 rows x [rows, W] over the row ranges
    [bounds[f], bounds[f + 1]) (host ints, nondecreasing), divided by `divisor`:
    [len(bounds) - 1, W] fp32, in a fixed order (reproducible run to run).  divisor =
    tokens per frame gives the frame mean (branch.py:450-452); 1 the sums of a sequence
    shard (ulysses_runtime.py:606-635).  One native launch (vdn_frame_sums)."""
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be bf16 [rows, W] with unit column stride")
    frames = len(bounds) - 1
    if out is None:
        out = torch.empty(frames, x.shape[1], device=x.device, dtype=torch.float32)
    if out.shape != (frames, x.shape[1]) or out.dtype != torch.float32 or not out.is_contiguous():
        raise ValueError("out must be contiguous fp32 [frames, W]")
    _lib.require_device(x)
    buf = (_lib.C.c_int32 * (frames + 1))(*[int(b) for b in bounds])
    _lib.call("vdn_frame_sums", _lib.ptr(x), x.stride(0), x.shape[0], x.shape[1], buf, frames, float(divisor),
              _lib.ptr(out), _lib.stream_of(x.device))
    return out


class FrameKDAAlpha(nn.Module):
    """alpha = exp(-exp(A_log) * softplus(up(down(mean)) + dt_bias)), fp32 (layers.py:12-69)."""

    def __init__(self, hidden_size, num_heads, head_dim, bottleneck=None):
        super().__init__()
        self.num_heads, self.head_dim = num_heads, head_dim
        bottleneck = bottleneck or head_dim
        self.down = nn.Linear(hidden_size, bottleneck, bias=False)
        self.up = nn.Linear(bottleneck, num_heads * head_dim, bias=False)
        self.A_log = nn.Parameter(torch.log(torch.empty(num_heads, dtype=torch.float32).uniform_(1, 16)))
        dt = torch.exp(torch.rand(num_heads * head_dim, dtype=torch.float32)
                       * (math.log(0.1) - math.log(0.001)) + math.log(0.001)).clamp(min=1e-4)
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))

    def forward_native(self, frame_mean_x, heads=None):
        """The same alpha from two library launches (vdn_frame_alpha), no host sync."""
        if heads is None:
            heads = slice(0, self.num_heads)
        rows = slice(heads.start * self.head_dim, heads.stop * self.head_dim)
        n_heads = heads.stop - heads.start
        fm = frame_mean_x.float().contiguous()
        f, hidden = fm.shape
        down = self.down.weight.float().contiguous()
        up = self.up.weight[rows].float().contiguous()
        dt = self.dt_bias[rows].float().contiguous()
        a_log = self.A_log[heads].float().contiguous()
        r = down.shape[0]
        scratch = torch.empty(f, r, device=fm.device, dtype=torch.float32)
        out = torch.empty(f, n_heads, self.head_dim, device=fm.device, dtype=torch.float32)
        _lib.require_device(fm, "frame_mean")
        _lib.call("vdn_frame_alpha", _lib.ptr(fm), f, hidden, _lib.ptr(down), r, _lib.ptr(up),
                  _lib.ptr(dt), _lib.ptr(a_log), n_heads, self.head_dim, _lib.ptr(scratch),
                  _lib.ptr(out), _lib.stream_of(fm.device))
        return out

    def forward(self, frame_mean_x, heads=None):
        if heads is None:
            up_w, dt_bias, a_log, n_heads = self.up.weight, self.dt_bias, self.A_log, self.num_heads
        else:
            rows = slice(heads.start * self.head_dim, heads.stop * self.head_dim)
            up_w, dt_bias, a_log = self.up.weight[rows], self.dt_bias[rows], self.A_log[heads]
            n_heads = heads.stop - heads.start
        with torch.autocast(device_type=frame_mean_x.device.type, enabled=False):
            delta = F.linear(frame_mean_x.float(), self.down.weight.float())
            delta = F.linear(delta, up_w.float()) + dt_bias.float()
            scale = torch.exp(a_log.float())[:, None]
            delta = delta.view(-1, n_heads, self.head_dim)
            return torch.exp(-scale * F.softplus(delta))


# ------------------------------------------------------------------ stage ops
def _bf16_cuda(t, name):
    if not isinstance(t, torch.Tensor) or t.dtype != torch.bfloat16 or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA BF16 tensor")
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must have a contiguous last dimension")
    _lib.require_device(t, name)


def vda_statistics(key, value, beta, *, features_applied=True):
    """A, B [F, H, d, d] fp32 from [F, H, S, d] bf16 k / v and [F, H, S] bf16 beta.

    features_applied=True: k / v are already SiLU(+L2) features (paper_statistics,
    paper_stack.py:86-110); False: raw projections, features applied in-kernel.
    """
    _bf16_cuda(key, "key")
    _bf16_cuda(value, "value")
    _bf16_cuda(beta.unsqueeze(-1), "beta")
    if key.ndim != 4 or value.shape != key.shape or beta.shape != key.shape[:-1]:
        raise ValueError("statistics require [F,H,S,d] k/v and [F,H,S] beta")
    f, h, s, d = key.shape
    a = torch.empty((f, h, d, d), dtype=torch.float32, device=key.device)
    b = torch.empty_like(a)
    ks, vs, bs = key.stride(), value.stride(), beta.stride()
    _lib.call("vdn_vda_statistics", _lib.ptr(key), ks[0], ks[2], ks[1], _lib.ptr(value), vs[0],
              vs[2], vs[1], _lib.ptr(beta), bs[0], bs[2], bs[1], int(features_applied), f, s, h, d,
              _lib.ptr(a), _lib.ptr(b), _lib.stream_of(key.device))
    return a, b


def vda_scan(transitions, injections, seed=None):
    """Full forward / reverse state banks [F, H, d, d] fp32 (scan.py:270-355)."""
    for t, n in ((transitions, "transitions"), (injections, "injections")):
        if t.dtype != torch.float32 or not t.is_cuda or not t.is_contiguous():
            raise ValueError(f"{n} must be contiguous CUDA fp32")
    if transitions.shape != injections.shape or transitions.ndim != 4:
        raise ValueError("matching [F,H,d,d] factors required")
    f, h, d, _ = transitions.shape
    if seed is not None:
        if seed.shape != (h, d, d) or seed.dtype != torch.float32:
            raise ValueError("seed must be fp32 [H,d,d]")
        seed = seed.contiguous()
    _lib.require_device(transitions)
    prefix = torch.empty_like(transitions)
    suffix = torch.empty_like(transitions)
    _lib.call("vdn_vda_scan", _lib.ptr(transitions), _lib.ptr(injections), _lib.ptr(seed), f, h, d,
              _lib.ptr(prefix), _lib.ptr(suffix), _lib.stream_of(transitions.device))
    return prefix, suffix


SPLIT_INVERSE_BYTES = 3 * 2 * 128 * 128   # three bf16 operand planes per 128 x 128 inverse


def vda_factor_inverse(A):
    """(I + A)^-1 of [..., 128, 128] fp32 matrices as three bf16 tensor-core operand
    planes per matrix (uint8 [..., 98304]): the factor stage of the d = 128 forward."""
    if A.dtype != torch.float32 or not A.is_cuda or A.shape[-2:] != (128, 128):
        raise ValueError("A must be CUDA fp32 [..., 128, 128]")
    _lib.require_device(A)
    A = A.contiguous()
    n = A.numel() // (128 * 128)
    planes = torch.empty(*A.shape[:-2], SPLIT_INVERSE_BYTES, dtype=torch.uint8, device=A.device)
    _lib.call("vdn_vda_factor_inverse", _lib.ptr(A), n, _lib.ptr(planes), _lib.stream_of(A.device))
    return planes


def split_inverse_values(planes):
    """Decode the planes of vda_factor_inverse back to the fp32 matrices [..., 128, 128]
    (un-swizzle the 16-byte chunks, sum the three bf16 parts: exact)."""
    lead = planes.shape[:-1]
    raw = planes.reshape(-1, 3, 2, 128, 8, 16).view(torch.int16)          # [n, part, half, row, chunk, 8]
    rows = torch.arange(128, device=planes.device)
    logical = torch.arange(8, device=planes.device)[None, :] ^ (rows[:, None] & 7)   # physical chunk
    idx = logical[None, None, None, :, :, None].expand(raw.shape[0], 3, 2, 128, 8, 8)
    ordered = torch.gather(raw, 4, idx)                                    # [n, part, half, row, chunk, 8]
    vals = ordered.view(torch.bfloat16).float()
    full = vals.permute(0, 1, 3, 2, 4, 5).reshape(-1, 3, 128, 128).sum(1)
    return full.reshape(*lead, 128, 128)


def vda_scan_tc(planes, B, alpha, seed=None):
    """Forward / reverse banks [F, H, 128, 128] fp32 from split inverses [F, H, 98304],
    B [F, H, 128, 128] and alpha [F, H, 128]: P_f = (P_{f-1} diag(alpha_f) + B_f) inv_f
    on the tensor cores (the d = 128 scan of vda_forward).  B fp32, or bf16 (the form
    the forward passes: B_f then reaches the kernel by TMA)."""
    f, h = B.shape[:2]
    if (B.shape != (f, h, 128, 128) or B.dtype not in (torch.float32, torch.bfloat16)
            or planes.shape != (f, h, SPLIT_INVERSE_BYTES)):
        raise ValueError("B must be fp32 or bf16 [F,H,128,128] and planes uint8 [F,H,98304]")
    if alpha.shape != (f, h, 128):
        raise ValueError("alpha must be [F,H,128]")
    _lib.require_device(B)
    if seed is not None:
        seed = seed.float().contiguous()
        if seed.shape != (h, 128, 128):
            raise ValueError("seed must be fp32 [H,128,128]")
    prefix = torch.empty(B.shape, dtype=torch.float32, device=B.device)
    suffix = torch.empty_like(prefix)
    status = torch.zeros(1, dtype=torch.int32, device=B.device)
    entry = "vdn_vda_scan_tc_bf16" if B.dtype == torch.bfloat16 else "vdn_vda_scan_tc"
    _lib.call(entry, _lib.ptr(planes.contiguous()), _lib.ptr(B.contiguous()),
              _lib.ptr(alpha.float().contiguous()), _lib.ptr(seed), f, h, _lib.ptr(prefix), _lib.ptr(suffix),
              _lib.ptr(status), _lib.stream_of(B.device))
    if int(status.item()):
        raise RuntimeError("VDA tensor-core scan wait timed out on the device")
    return prefix, suffix


def _bounds_buffer(bounds, frames):
    if len(bounds) != frames or frames < 1 or frames > MAX_FRAMES:
        raise ValueError(f"one bound per frame required (1..{MAX_FRAMES} frames)")
    flat = []
    for f, (lo, hi) in enumerate(bounds):
        lo, hi = int(lo), int(hi)
        if not lo <= f <= hi:
            raise ValueError("each inclusive window must contain its query frame")
        flat += [lo, hi]
    return (_lib.C.c_int32 * len(flat))(*flat)


def vda_gather(prefix, suffix, alpha, bounds, seed=None, out_dtype=torch.bfloat16, bridge=True):
    """Window-complement state per frame, decayed in (scan.py:361-496)."""
    f, h, d, _ = prefix.shape
    if alpha.shape != (f, h, d) or alpha.dtype != torch.float32:
        raise ValueError("alpha must be fp32 [F,H,d]")
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out_dtype must be bf16 or fp32")
    _lib.require_device(prefix)
    out = torch.empty((f, h, d, d), dtype=out_dtype, device=prefix.device)
    buf = _bounds_buffer(bounds, f)
    _lib.call("vdn_vda_gather", _lib.ptr(prefix.contiguous()), _lib.ptr(suffix.contiguous()),
              _lib.ptr(alpha.contiguous()), buf, _lib.ptr(None if seed is None else seed.contiguous()),
              int(bool(bridge)), f, h, d, _lib.ptr(out), _lib.dtype_code(out_dtype),
              _lib.stream_of(prefix.device))
    return out


def vda_text_seed(text_k_raw, text_v_raw, text_beta, scale=0.5):
    """scale * S_text [H, d, d] fp32: the prompt as one chunk into a zero state (branch.py:190-238)."""
    length, h, d = text_k_raw.shape
    k = text_k_raw.unsqueeze(0).permute(0, 2, 1, 3)   # [1, H, L, d] view
    v = text_v_raw.unsqueeze(0).permute(0, 2, 1, 3)
    b = text_beta.reshape(1, length, h).permute(0, 2, 1)
    a, bb = vda_statistics(k, v, b, features_applied=False)
    _, inj = paper_delta_factors(a, bb)
    return inj[0] * scale


def vda_forward(q, k, v, beta, gate, alpha, bounds, num_frames, tokens_per_frame, norm_weight,
                eps=1e-6, seed=None, bridge=True):
    """The native branch body over [F*S, H, d] raw q / k / v. Returns [F*S, H*d] bf16."""
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (gate, "gate")):
        _bf16_cuda(t, n)
    if q.stride() != k.stride() or q.stride() != v.stride():
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    f, s = num_frames, tokens_per_frame
    n, h, d = q.shape
    if n != f * s or k.shape != q.shape or v.shape != q.shape or gate.shape != q.shape:
        raise ValueError("q/k/v/gate must be [F*S, H, d]")
    if beta.shape != (n, h) or beta.dtype != torch.bfloat16:
        raise ValueError("beta must be bf16 [F*S, H]")
    alpha = alpha.float().contiguous()
    if alpha.shape != (f, h, d):
        raise ValueError("alpha must be [F, H, d]")
    w = norm_weight.float().contiguous()
    if seed is not None:
        seed = seed.float().contiguous()
        if seed.shape != (h, d, d):
            raise ValueError("seed must be [H, d, d]")
    _lib.require_device(q, "q")
    out = torch.empty((n, h * d), dtype=torch.bfloat16, device=q.device)
    ws_bytes = _lib.load().vdn_vda_workspace_size(f, s, h, d)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    buf = _bounds_buffer(bounds, f)
    qs = q.stride()
    _lib.call("vdn_vda_forward", _lib.ptr(q), _lib.ptr(k), _lib.ptr(v), qs[0], qs[1], _lib.ptr(beta),
              beta.stride(0), beta.stride(1), _lib.ptr(gate), gate.stride(0), gate.stride(1),
              _lib.ptr(alpha), _lib.ptr(w), float(eps), buf, _lib.ptr(seed), int(bool(bridge)),
              f, s, h, d, _lib.ptr(out), _lib.ptr(ws), ws_bytes, _lib.stream_of(q.device))
    return out


# --------------------------------------------------------------------- module
class BidirectionalLinearBranch(nn.Module):
    """NoPE linear-attention branch, native B200 body (branch.py:47-402).

    Supports the released-checkpoint rule (delta_rule="vdn_solve", a_fp32) with
    bridge "alpha" or "none", the text seed, the anchor frames and the separable
    short conv (short_conv=("k", "v") as released; any subset of q / k / v).
    """

    TEXT_STATE_SCALE = 0.5

    def __init__(self, hidden_size, num_heads, head_dim, delta_rule="vdn_solve",
                 gate_bottleneck=None, bridge="alpha", a_fp32=True, short_conv=()):
        super().__init__()
        if delta_rule != "vdn_solve":
            raise ValueError("the B200 branch implements delta_rule='vdn_solve'")
        if not a_fp32:
            raise ValueError("the B200 branch computes A in fp32 (a_fp32=True)")
        if bridge not in BRIDGE_MODES:
            raise ValueError(f"bridge must be one of {BRIDGE_MODES}")
        if head_dim not in (64, 128):
            raise ValueError("head_dim must be 64 or 128")
        targets = tuple(short_conv) if isinstance(short_conv, (list, tuple)) else None
        if targets is None or any(t not in ("q", "k", "v") for t in targets) or len(set(targets)) != len(targets):
            raise ValueError(f"short_conv={short_conv!r}; expected a distinct subset of ('q', 'k', 'v')")
        self.num_heads, self.head_dim = num_heads, head_dim
        self.bridge = bridge
        self.a_fp32 = a_fp32
        self.delta_rule = delta_rule
        # None rather than a disabled module when off, so conv-less checkpoints keep
        # their exact parameter set (branch.py:68-78).
        from .short_conv import LinearAttentionSepConv
        self.short_conv = LinearAttentionSepConv(num_heads * head_dim, targets) if targets else None
        self.alpha = FrameKDAAlpha(hidden_size, num_heads, head_dim)
        self.beta_proj = nn.Linear(hidden_size, num_heads, bias=False)
        self.output_gate = OutputGate(hidden_size, num_heads, head_dim,
                                      bottleneck=gate_bottleneck or head_dim, init="random")
        self.norm = RMSNorm(head_dim)

    def _validate_sharded(self, heads, beta, gate, frame_mean, text_beta, text_qkv_raw):
        if heads is not None:
            if (not isinstance(heads, slice) or heads.step not in (None, 1)
                    or not isinstance(heads.start, int) or not isinstance(heads.stop, int)
                    or not 0 <= heads.start < heads.stop <= self.num_heads):
                raise ValueError("heads must be a bounded contiguous slice within num_heads")
            if beta is None or gate is None or frame_mean is None:
                raise ValueError("head-sharded calls require beta, gate, and frame_mean")
            if text_qkv_raw is not None and text_beta is None:
                raise ValueError("head-sharded text_qkv_raw requires text_beta")

    def forward(self, xv, num_frames, tokens_per_frame, bounds, qkv_raw, frame_size=None,
                skip_ends=False, text_x=None, text_qkv_raw=None, inference=False, heads=None,
                beta=None, gate=None, frame_mean=None, text_beta=None):
        """Everything the softmax window cannot see, for every video token (branch.py:256-402).

        Returns [F*S, H_local*d] bf16; anchor rows are exact zeros when skip_ends.
        """
        if torch.is_grad_enabled():
            raise RuntimeError("the B200 VDA branch is inference-only; call it under torch.no_grad()")
        if any(t.device.type != "cuda" or t.dtype != torch.bfloat16 for t in qkv_raw):
            raise ValueError("the B200 VDA branch requires CUDA BF16 Q/K/V")
        self._validate_sharded(heads, beta, gate, frame_mean, text_beta, text_qkv_raw)
        if self.short_conv is not None and frame_size is None:
            raise ValueError("short_conv needs the spatial grid; pass frame_size=(H, W)")
        n_heads = self.num_heads if heads is None else heads.stop - heads.start
        ref = xv if xv is not None else gate
        f, s = num_frames, tokens_per_frame
        if not skip_ends:
            return self._readout(xv, f, s, bounds, qkv_raw, text_x, text_qkv_raw, heads, beta,
                                 gate, frame_mean, text_beta, frame_size)
        if f <= 2:
            return ref.new_zeros(f * s, n_heads * self.head_dim, dtype=torch.bfloat16)
        inner = slice(s, (f - 1) * s)
        readout = self._readout(
            None if xv is None else xv[inner], f - 2, s,
            [(lo - 1, hi - 1) for lo, hi in bounds[1:f - 1]], tuple(t[inner] for t in qkv_raw),
            text_x, text_qkv_raw, heads, None if beta is None else beta[inner],
            None if gate is None else gate[inner], None if frame_mean is None else frame_mean[1:-1],
            text_beta, frame_size)
        out = readout.new_empty(f * s, readout.shape[-1])
        out[:s].zero_()
        out[(f - 1) * s:].zero_()
        out[inner] = readout
        return out

    def _readout(self, xv, f, s, bounds, qkv_raw, text_x, text_qkv_raw, heads, beta, gate,
                 frame_mean, text_beta, frame_size=None):
        h = self.num_heads if heads is None else heads.stop - heads.start
        d = self.head_dim
        q, k, v = qkv_raw
        if self.short_conv is not None:  # video rows only; the prompt has no grid
            q, k, v = (self.short_conv.apply(name, t, f, frame_size, heads=heads)
                       for name, t in zip(("q", "k", "v"), (q, k, v)))
        if beta is None:
            beta = torch.sigmoid(self.beta_proj(xv))
        beta = beta.to(torch.bfloat16).reshape(f * s, h)
        if gate is None:
            gate = self.output_gate(xv)
        gate = gate.to(torch.bfloat16).reshape(f * s, h, d)
        if gate.stride(-1) != 1:
            gate = gate.contiguous()
        if frame_mean is None:
            frame_mean = xv.view(f, s, -1).mean(dim=1, dtype=torch.float32)
        alpha = self.alpha(frame_mean, heads=heads).float()
        seed = None
        if text_x is not None or text_beta is not None:
            if text_qkv_raw is None or text_qkv_raw[1].shape[0] < 1:
                raise ValueError("prompt inputs require nonempty text QKV")
            tb = text_beta if text_beta is not None else torch.sigmoid(self.beta_proj(text_x))
            tb = tb.to(torch.bfloat16).reshape(-1, h)
            seed = vda_text_seed(text_qkv_raw[1], text_qkv_raw[2], tb, self.TEXT_STATE_SCALE)
        return vda_forward(q, k, v, beta, gate, alpha, bounds, f, s, self.norm.weight,
                           self.norm.eps, seed=seed, bridge=self.bridge == "alpha")
