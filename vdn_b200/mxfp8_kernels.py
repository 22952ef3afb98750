"""Fused MXFP8 producers and the device finite predicate.

Mirrors ec-jt/vdn src/models/ops/mxfp8_kernels.py (launch_quantize,
launch_swiglu_quantize, launch_prenorm_quantize, finite_parts) on sm_100a
kernels of libvdn_b200, plus launch_gelu_quantize: the same producer for a GELU
feed-forward (the block geometry this build targets uses GELU, the reference
only ships SwiGLU).
"""
from __future__ import annotations

import torch

from . import _lib
from .mxfp8_quant import launch_quantize, padded_shape, scale_numel

__all__ = ["launch_quantize", "launch_swiglu_quantize", "launch_gelu_quantize",
           "launch_prenorm_quantize", "finite_parts"]


def _act_quantize(act: int, x: torch.Tensor, k: int):
    _lib.require_device(x, "activation")
    if x.dtype != torch.bfloat16 or x.stride(-1) != 1:
        raise ValueError("expected CUDA BF16 rows with contiguous K")
    r = x.shape[0]
    rp, kp = padded_shape(r, k)
    q = torch.empty((rp, kp), dtype=torch.uint8, device=x.device)
    s = torch.empty(scale_numel(r, k), dtype=torch.uint8, device=x.device)
    bad = torch.zeros(1, dtype=torch.int32, device=x.device)
    _lib.call("vdn_mxfp8_act_quantize", act, _lib.ptr(x), r, k, x.stride(0) if r else x.shape[1],
              _lib.ptr(q), _lib.ptr(s), _lib.ptr(bad), _lib.stream_of(x.device))
    return q, s, bad == 0


def launch_swiglu_quantize(x: torch.Tensor):
    """[rows, 2K] (a | g) -> MXFP8 of bf16(a * silu(g)), plus a device finite flag."""
    r, twice_k = x.shape
    if twice_k % 2:
        raise ValueError("expected an even projection width")
    return _act_quantize(_lib.ACT_SWIGLU, x, twice_k // 2)


def launch_gelu_quantize(x: torch.Tensor, *, approximate: str = "tanh"):
    """[rows, K] -> MXFP8 of bf16(gelu(x)), plus a device finite flag."""
    act = {"tanh": _lib.ACT_GELU_TANH, "none": _lib.ACT_GELU_ERF}.get(approximate)
    if act is None:
        raise ValueError("approximate must be 'tanh' or 'none'")
    return _act_quantize(act, x, x.shape[1])


def launch_prenorm_quantize(x, weight, eps, scale, shift, indices, *, write_bf16):
    """RMSNorm * w * (1 + scale[idx]) + shift[idx] -> (bf16 | None, q, s, finite[RP])."""
    _lib.require_device(x, "hidden")
    r, k = x.shape
    if x.dtype != torch.bfloat16 or x.stride(-1) != 1:
        raise ValueError("expected CUDA BF16 hidden with contiguous K")
    if scale.dtype != torch.bfloat16 or shift.dtype != torch.bfloat16:
        raise ValueError("AdaLN tables must be BF16")
    if scale.stride(-1) != 1 or shift.stride(-1) != 1 or weight.stride(-1) != 1:
        raise ValueError("AdaLN tables and weight need a contiguous last dimension")
    indices = indices.to(torch.int64).contiguous()
    rp, kp = padded_shape(r, k)
    q = torch.empty((rp, kp), dtype=torch.uint8, device=x.device)
    s = torch.empty(scale_numel(r, k), dtype=torch.uint8, device=x.device)
    y = torch.empty((r, k), dtype=torch.bfloat16, device=x.device) if write_bf16 else None
    finite = torch.empty(rp, dtype=torch.bool, device=x.device)
    _lib.call("vdn_mxfp8_prenorm_quantize", _lib.ptr(x), r, k, x.stride(0) if r else k,
              _lib.ptr(weight), _lib.dtype_code(weight.dtype), float(eps), _lib.ptr(scale),
              scale.stride(0), _lib.ptr(shift), shift.stride(0), _lib.ptr(indices), _lib.ptr(y),
              _lib.ptr(q), _lib.ptr(s), _lib.ptr(finite), _lib.stream_of(x.device))
    return y, q, s, finite


def finite_parts(x: torch.Tensor, mode: int = 0) -> torch.Tensor:
    """One bool per 4096 elements: floats (0), E4M3 codes (1) or E8M0 bytes (2)."""
    _lib.require_device(x)
    x = x.contiguous()
    n = x.numel()
    parts = torch.empty((n + 4095) // 4096, dtype=torch.bool, device=x.device)
    dtype = _lib.DTYPE_F32 if mode else _lib.dtype_code(x.dtype)
    if mode and x.dtype != torch.uint8:
        raise TypeError("modes 1 and 2 read uint8 bytes")
    _lib.call("vdn_finite_parts", _lib.ptr(x), n, dtype, int(mode), _lib.ptr(parts),
              _lib.stream_of(x.device))
    return parts
