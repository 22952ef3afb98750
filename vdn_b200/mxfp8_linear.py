"""MXFP8 linears on the sm_100a block-scaled tcgen05 GEMM.

Public surface of ec-jt/vdn src/models/ops/mxfp8_linear.py (SUPPORTED_ROLES,
MXFP8Linear with uint8 buffers weight_data / weight_scale and no .weight,
forward_quantized / forward, projection_features, project, project_to_out,
project_qkv, convert_linear_to_mxfp8), with the same argument meaning and the
same error types and messages.  The reference's GEMM is SM120-only
(F.scaled_mm); here every GEMM is vdn_mxfp8_gemm (tcgen05, kind::mxf8f6f4).

Design: a weight is packed once into a `_Packing` record (padded geometry,
codes, swizzled scales); one validation pass checks a prepared activation
against it; finite checks run as device predicates with a single host read per
call.  project_qkv shares one activation quantisation and, when every width is
a multiple of 128, runs ONE GEMM over the concatenated Q|K|V weight
(N = 3 x 5120 = 15360 in the target block).  Model conversion is planned in full
(role table walk, tied-weight count) before any module is replaced.
"""
from __future__ import annotations

import math
from collections import Counter
from typing import NamedTuple

import torch
from torch import nn

from . import _lib
from .mxfp8_kernels import finite_parts
from .mxfp8_quant import (padded_shape, quantize_activation, quantize_cpu, require_finite,
                          scale_numel)

# Role -> submodule path inside one transformer block (mxfp8_linear.py:17-25).
SUPPORTED_ROLES = {
    "q": "attn.orig.to_q",
    "k": "attn.orig.to_k",
    "v": "attn.orig.to_v",
    "softmax_out": "attn.orig.to_out.0",
    "linear_out": "attn.to_out_linear",
    "ff_up": "ff.net.0.proj",
    "ff_down": "ff.net.2",
}


def require_native_sm100(device):
    """RuntimeError unless `device` is an sm_100 CUDA device (no fallback)."""
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("native MXFP8 requires sm_100 CUDA execution; no fallback")
    _lib.require_device(torch.empty(0, device=device))


# One int32 status word per device: GEMM pipeline timeouts are reported there.
_STATUS: dict[int, torch.Tensor] = {}


def _status(device) -> torch.Tensor:
    idx = torch.cuda.current_device() if device.index is None else device.index
    word = _STATUS.get(idx)
    if word is None:
        word = _STATUS[idx] = torch.zeros(1, dtype=torch.int32, device=device)
    return word


def mxfp8_gemm(data, scales, weight_data, weight_scale, n, *, rows, bias=None, out=None):
    """y[:rows, :n] = bf16(dequant(data) dequant(weight)^T) (+ bias) on tcgen05."""
    m_pad, k_pad = data.shape
    n_pad, k_w = weight_data.shape
    if k_w != k_pad:
        raise ValueError("activation and weight K padding differ")
    y = torch.empty((rows, n), dtype=torch.bfloat16, device=data.device) if out is None else out
    if rows:
        _lib.call("vdn_mxfp8_gemm", _lib.ptr(data), _lib.ptr(scales), _lib.ptr(weight_data),
                  _lib.ptr(weight_scale), _lib.ptr(bias), m_pad, n, n_pad, k_pad, rows, _lib.ptr(y),
                  y.stride(0), _lib.ptr(_status(data.device)), _lib.stream_of(data.device))
    return y


def check_gemm_status(device) -> None:
    """Raise RuntimeError if a GEMM on `device` reported a pipeline timeout (host read)."""
    word = _status(torch.device(device))
    if int(word.item()):
        word.zero_()
        raise RuntimeError("MXFP8 GEMM pipeline wait timed out on the device")


class _Packing(NamedTuple):
    """Padded geometry of one packed weight: codes [n_pad, k_pad], scale bytes."""
    n: int
    k: int
    n_pad: int
    k_pad: int
    scale_bytes: int

    @classmethod
    def of(cls, n, k):
        n_pad, k_pad = padded_shape(n, k)
        return cls(n, k, n_pad, k_pad, scale_numel(n_pad, k_pad))


def _activation_rows(data, scales, weight_data, weight_scale, packing: _Packing, rows):
    """Check a prepared activation against a packed weight; return the output row count."""
    operands = (data, scales, weight_data, weight_scale)
    if any(t.dtype != torch.uint8 or not t.is_contiguous() or t.device != data.device for t in operands):
        raise ValueError("MXFP8 data/scales must be contiguous uint8 on the same CUDA device")
    if data.ndim != 2 or data.shape[1] != packing.k_pad or data.shape[0] % 128:
        raise ValueError("invalid padded activation shape")
    if (tuple(weight_data.shape) != (packing.n_pad, packing.k_pad)
            or tuple(weight_scale.shape) != (packing.scale_bytes,)):
        raise ValueError("invalid compressed weight layout")
    if tuple(scales.shape) != (scale_numel(data.shape[0], packing.k_pad),):
        raise ValueError("invalid activation scale layout")
    out_rows = data.shape[0] if rows is None else rows
    if not 0 <= out_rows <= data.shape[0]:
        raise ValueError("invalid output row count")
    return out_rows


class MXFP8Linear(nn.Module):
    """Inference-only effective weight stored as two uint8 buffers (mxfp8_linear.py:36-102):
    `weight_data` (E4M3 codes, padded to 128) and `weight_scale` (E8M0, SWIZZLE_32_4_4).

    There is no .weight; use forward_quantized / forward / projection_features.
    """

    def __init__(self, linear: nn.Linear, *, chunk_rows=128, check_finite=True):
        super().__init__()
        if type(check_finite) is not bool:
            raise ValueError("check_finite must be a bool")
        if type(linear) is not nn.Linear:
            raise TypeError("MXFP8 requires an ordinary merged nn.Linear")
        bias = linear.bias
        codes, scale_bytes = quantize_cpu(linear.weight, chunk_rows=chunk_rows)
        if bias is not None and not bias.is_meta:
            require_finite(bias, "bias")
        self.in_features, self.out_features = linear.in_features, linear.out_features
        self.check_finite = check_finite
        self.register_buffer("weight_data", codes)
        self.register_buffer("weight_scale", scale_bytes)
        frozen = None if bias is None else nn.Parameter(bias.detach(), requires_grad=False)
        self.register_parameter("bias", frozen)
        self.eval()

    @property
    def packing(self) -> _Packing:
        return _Packing.of(self.out_features, self.in_features)

    def _bias_bf16(self):
        return None if self.bias is None else self.bias.to(torch.bfloat16).contiguous()

    @torch.no_grad()
    def forward_quantized(self, data, scales, *, rows=None, out_dtype=torch.bfloat16):
        """Consume padded uint8 codes and swizzled scales, return cropped bf16 [rows, N]."""
        if self.training or out_dtype != torch.bfloat16:
            raise ValueError("MXFP8 supports eval BF16 output only")
        require_native_sm100(data.device)
        rows = _activation_rows(data, scales, self.weight_data, self.weight_scale, self.packing, rows)
        if rows == 0:
            return torch.empty((0, self.out_features), device=data.device, dtype=out_dtype)
        if not self.check_finite:
            return mxfp8_gemm(data, scales, self.weight_data, self.weight_scale, self.out_features,
                              rows=rows, bias=self._bias_bf16())
        inputs_ok = torch.cat((finite_parts(data, 1), finite_parts(scales, 2))).all()
        y = mxfp8_gemm(data, scales, self.weight_data, self.weight_scale, self.out_features,
                       rows=rows, bias=self._bias_bf16())
        verdict = torch.stack((inputs_ok, finite_parts(y).all())).cpu()   # the one host read
        check_gemm_status(data.device)
        if not bool(verdict[0]):
            raise ValueError("nonfinite MXFP8 prepared activation")
        if not bool(verdict[1]):
            raise ValueError("nonfinite MXFP8 result")
        return y

    @torch.no_grad()
    def forward(self, x):
        if x.ndim < 2 or x.shape[-1] != self.in_features or x.requires_grad:
            raise ValueError("MXFP8 expects inference activation [...,in_features]")
        lead = x.shape[:-1]
        flat = x.reshape(math.prod(lead), self.in_features).contiguous()
        data, scales = quantize_activation(flat, check_finite=self.check_finite)
        return self.forward_quantized(data, scales, rows=flat.shape[0]).view(*lead, self.out_features)


# ------------------------------------------------------------- projection helpers
_PROJECTIONS = (nn.Linear, MXFP8Linear)


def projection_features(module):
    """(in_features, out_features) of a plain or MXFP8 projection; TypeError otherwise."""
    if isinstance(module, _PROJECTIONS):
        return module.in_features, module.out_features
    raise TypeError("unsupported projection module")


def project(module, x):
    """Apply a projection through its module (never through a .weight read)."""
    projection_features(module)
    return module(x)


def project_to_out(to_out, x):
    """to_out as a bare projection, or a (projection, dropout) pair."""
    if not isinstance(to_out, (nn.ModuleList, nn.Sequential, list, tuple)):
        return project(to_out, x)
    if len(to_out) != 2:
        raise ValueError("expected projection/dropout pair")
    projection, dropout = to_out
    return dropout(project(projection, x))


def _fused_qkv_weights(projections):
    """Concatenated Q|K|V codes, scales and bias, cached on the first projection."""
    key = tuple((id(p.weight_data), p.weight_data.data_ptr(), id(p.weight_scale)) for p in projections)
    cache = getattr(projections[0], "_fused_qkv", None)
    if cache is not None and cache[0] == key:
        return cache[1]
    data = torch.cat([p.weight_data for p in projections])
    scales = torch.cat([p.weight_scale for p in projections])
    bias = None
    if any(p.bias is not None for p in projections):
        bias = torch.cat([p._bias_bf16() if p.bias is not None else
                          torch.zeros(p.out_features, dtype=torch.bfloat16, device=data.device)
                          for p in projections])
    fused = (data, scales, bias)
    object.__setattr__(projections[0], "_fused_qkv", (key, fused))
    return fused


def project_qkv(projections, x):
    """Q, K, V of x sharing one activation quantisation (mxfp8_linear.py:127-142)."""
    if len(projections) != 3:
        raise ValueError("expected Q, K, V")
    kinds = {isinstance(p, MXFP8Linear) for p in projections}
    if kinds == {False}:
        return tuple(project(p, x) for p in projections)
    if kinds == {True, False}:
        raise ValueError("mixed QKV precision is not supported")
    if x.requires_grad or any(p.in_features != x.shape[-1] for p in projections):
        raise ValueError("invalid inference QKV input")
    lead = x.shape[:-1]
    flat = x.reshape(math.prod(lead), x.shape[-1]).contiguous()
    checked = any(p.check_finite for p in projections)
    data, scales = quantize_activation(flat, check_finite=checked)
    widths = [p.out_features for p in projections]
    if not checked and all(w % 128 == 0 for w in widths):
        wd, ws, bias = _fused_qkv_weights(projections)
        y = mxfp8_gemm(data, scales, wd, ws, sum(widths), rows=flat.shape[0], bias=bias)
        return tuple(part.view(*lead, w) for part, w in zip(y.split(widths, dim=-1), widths))
    return tuple(p.forward_quantized(data, scales, rows=flat.shape[0]).view(*lead, p.out_features)
                 for p in projections)


# ------------------------------------------------------------------- conversion
class _Target(NamedTuple):
    block: int
    role: str
    path: str
    parent: nn.Module
    attr: str
    linear: nn.Linear


def _plan_conversion(model) -> list[_Target]:
    """Every (block, role) target of the role table, validated before anything changes:
    each must be an ordinary nn.Linear on the CPU or meta device whose weight no other
    parameter slot of the model shares."""
    slots = Counter(id(p) for _, p in model.named_parameters(remove_duplicate=False))
    taken: set[int] = set()
    plan = []
    for index, block in enumerate(model.transformer_blocks):
        for role, path in SUPPORTED_ROLES.items():
            module = block.get_submodule(path)
            if type(module) is not nn.Linear or module.weight.device.type not in ("cpu", "meta"):
                raise ValueError(f"{index}:{role} requires a merged CPU/meta nn.Linear")
            wid = id(module.weight)
            if wid in taken or slots[wid] != 1:
                raise ValueError("tied MXFP8 target weights are unsupported")
            taken.add(wid)
            parent_path, attr = path.rsplit(".", 1)
            plan.append(_Target(index, role, path, block.get_submodule(parent_path), attr, module))
    return plan


def convert_linear_to_mxfp8(model, *, enabled=False, chunk_rows=128, check_finite=True):
    """Replace the seven projection roles of every transformer block with MXFP8Linear
    (mxfp8_linear.py:145-180).  Off by default (returns []); refuses a model in training
    mode, a role that is not a merged CPU/meta nn.Linear, and tied target weights, all
    before any module is replaced.  Returns one record per converted module."""
    if type(enabled) is not bool or type(check_finite) is not bool:
        raise ValueError("enabled and check_finite must be booleans")
    if not enabled:
        return []
    if model.training:
        raise ValueError("convert an eval model after effective-weight merging")
    plan = _plan_conversion(model)
    records = []
    for t in plan:
        records.append(dict(block=t.block, role=t.role, module=f"transformer_blocks.{t.block}.{t.path}",
                            in_features=t.linear.in_features, out_features=t.linear.out_features))
        setattr(t.parent, t.attr, MXFP8Linear(t.linear, chunk_rows=chunk_rows, check_finite=check_finite))
    return records
