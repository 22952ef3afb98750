"""MXFP8 linears on the sm_100a block-scaled tcgen05 GEMM.

Mirrors ec-jt/vdn src/models/ops/mxfp8_linear.py: SUPPORTED_ROLES,
MXFP8Linear (uint8 buffers weight_data / weight_scale, no .weight,
forward_quantized / forward), projection_features, project, project_to_out,
project_qkv and convert_linear_to_mxfp8, with the same errors.  The reference's
GEMM is SM120-only (F.scaled_mm); here the GEMM is vdn_mxfp8_gemm.  Finite
checks run as device predicates and cost one host read per call instead of
three.  project_qkv shares one activation quantisation and, when every
projection width is a multiple of 128, runs ONE GEMM over the concatenated
Q|K|V weight (N = 3 x 5120 = 15360 in the target block).
"""
from __future__ import annotations

import math

import torch
from torch import nn

from . import _lib
from .mxfp8_kernels import finite_parts
from .mxfp8_quant import (padded_shape, quantize_activation, quantize_cpu, require_finite,
                          scale_numel)

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


_STATUS: dict[int, torch.Tensor] = {}


def _status(device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _STATUS:
        _STATUS[idx] = torch.zeros(1, dtype=torch.int32, device=device)
    return _STATUS[idx]


def mxfp8_gemm(data, scales, weight_data, weight_scale, n, *, rows, bias=None, out=None):
    """y[:rows, :n] = bf16(dequant(data) dequant(weight)^T) (+ bias) on tcgen05."""
    mp, kp = data.shape
    np_, kw = weight_data.shape
    if kw != kp:
        raise ValueError("activation and weight K padding differ")
    y = out if out is not None else torch.empty((rows, n), dtype=torch.bfloat16, device=data.device)
    if rows == 0:
        return y
    status = _status(data.device)
    _lib.call("vdn_mxfp8_gemm", _lib.ptr(data), _lib.ptr(scales), _lib.ptr(weight_data),
              _lib.ptr(weight_scale), _lib.ptr(bias), mp, n, np_, kp, rows, _lib.ptr(y),
              y.stride(0), _lib.ptr(status), _lib.stream_of(data.device))
    return y


def check_gemm_status(device) -> None:
    """Raise RuntimeError if a GEMM on `device` reported a pipeline timeout (host read)."""
    st = _status(torch.device(device))
    if int(st.item()):
        st.zero_()
        raise RuntimeError("MXFP8 GEMM pipeline wait timed out on the device")


class MXFP8Linear(nn.Module):
    """Inference-only effective weight stored as two uint8 buffers (mxfp8_linear.py:36-102).

    There is no .weight; use forward_quantized / forward / projection_features.
    """

    def __init__(self, linear: nn.Linear, *, chunk_rows=128, check_finite=True):
        super().__init__()
        if type(check_finite) is not bool:
            raise ValueError("check_finite must be a bool")
        if type(linear) is not nn.Linear:
            raise TypeError("MXFP8 requires an ordinary merged nn.Linear")
        self.in_features, self.out_features = linear.in_features, linear.out_features
        self.check_finite = check_finite
        data, scales = quantize_cpu(linear.weight, chunk_rows=chunk_rows)
        if linear.bias is not None and not linear.bias.is_meta:
            require_finite(linear.bias, "bias")
        self.register_buffer("weight_data", data)
        self.register_buffer("weight_scale", scales)
        self.register_parameter("bias", None if linear.bias is None else
                                nn.Parameter(linear.bias.detach(), requires_grad=False))
        self.eval()

    def _bias_bf16(self):
        if self.bias is None:
            return None
        b = self.bias
        if b.dtype != torch.bfloat16:
            b = b.to(torch.bfloat16)
        return b.contiguous()

    @torch.no_grad()
    def forward_quantized(self, data, scales, *, rows=None, out_dtype=torch.bfloat16):
        """Consume padded uint8 codes and swizzled scales, return cropped bf16 [rows, N]."""
        if self.training or out_dtype != torch.bfloat16:
            raise ValueError("MXFP8 supports eval BF16 output only")
        require_native_sm100(data.device)
        tensors = (data, scales, self.weight_data, self.weight_scale)
        if any(t.dtype != torch.uint8 or not t.is_contiguous() or t.device != data.device for t in tensors):
            raise ValueError("MXFP8 data/scales must be contiguous uint8 on the same CUDA device")
        np_, kp = padded_shape(self.out_features, self.in_features)
        if data.ndim != 2 or data.shape[1] != kp or data.shape[0] % 128:
            raise ValueError("invalid padded activation shape")
        if self.weight_data.shape != (np_, kp) or self.weight_scale.shape != (scale_numel(np_, kp),):
            raise ValueError("invalid compressed weight layout")
        if scales.shape != (scale_numel(data.shape[0], kp),):
            raise ValueError("invalid activation scale layout")
        rows = data.shape[0] if rows is None else rows
        if not 0 <= rows <= data.shape[0]:
            raise ValueError("invalid output row count")
        if rows == 0:
            return torch.empty((0, self.out_features), device=data.device, dtype=out_dtype)
        if self.check_finite:
            pre = torch.cat((finite_parts(data, 1), finite_parts(scales, 2)))
        y = mxfp8_gemm(data, scales, self.weight_data, self.weight_scale, self.out_features,
                       rows=rows, bias=self._bias_bf16())
        if self.check_finite:
            post = finite_parts(y)
            ok = torch.stack((pre.all(), post.all())).cpu()
            check_gemm_status(data.device)
            if not bool(ok[0]):
                raise ValueError("nonfinite MXFP8 prepared activation")
            if not bool(ok[1]):
                raise ValueError("nonfinite MXFP8 result")
        return y

    @torch.no_grad()
    def forward(self, x):
        if x.ndim < 2 or x.shape[-1] != self.in_features or x.requires_grad:
            raise ValueError("MXFP8 expects inference activation [...,in_features]")
        rows = math.prod(x.shape[:-1])
        data, scales = quantize_activation(x.reshape(rows, self.in_features).contiguous(),
                                           check_finite=self.check_finite)
        return self.forward_quantized(data, scales, rows=rows).reshape(*x.shape[:-1], self.out_features)


def projection_features(module):
    if not isinstance(module, (nn.Linear, MXFP8Linear)):
        raise TypeError("unsupported projection module")
    return module.in_features, module.out_features


def project(module, x):
    projection_features(module)
    return module(x)


def project_to_out(to_out, x):
    if isinstance(to_out, (nn.ModuleList, nn.Sequential, list, tuple)):
        if len(to_out) != 2:
            raise ValueError("expected projection/dropout pair")
        return to_out[1](project(to_out[0], x))
    return project(to_out, x)


def _fused_qkv_weights(projections):
    """Concatenated Q|K|V codes, scales and bias, cached on the first projection."""
    key = tuple((id(p.weight_data), p.weight_data.data_ptr(), id(p.weight_scale)) for p in projections)
    cache = getattr(projections[0], "_fused_qkv", None)
    if cache is not None and cache[0] == key:
        return cache[1]
    data = torch.cat([p.weight_data for p in projections])
    scales = torch.cat([p.weight_scale for p in projections])
    biases = [p._bias_bf16() for p in projections]
    bias = None
    if any(b is not None for b in biases):
        bias = torch.cat([b if b is not None else torch.zeros(p.out_features, dtype=torch.bfloat16,
                                                              device=data.device)
                          for b, p in zip(biases, projections)])
    fused = (data, scales, bias)
    object.__setattr__(projections[0], "_fused_qkv", (key, fused))
    return fused


def project_qkv(projections, x):
    """Share one activation quantisation for three MXFP8 projections (mxfp8_linear.py:127-142)."""
    if len(projections) != 3:
        raise ValueError("expected Q, K, V")
    native = [isinstance(p, MXFP8Linear) for p in projections]
    if any(native) and not all(native):
        raise ValueError("mixed QKV precision is not supported")
    if not any(native):
        return tuple(project(p, x) for p in projections)
    if x.requires_grad or any(p.in_features != x.shape[-1] for p in projections):
        raise ValueError("invalid inference QKV input")
    rows = math.prod(x.shape[:-1])
    data, scales = quantize_activation(x.reshape(rows, x.shape[-1]).contiguous(),
                                       check_finite=any(p.check_finite for p in projections))
    widths = [p.out_features for p in projections]
    if all(w % 128 == 0 for w in widths) and not any(p.check_finite for p in projections):
        wd, ws, bias = _fused_qkv_weights(projections)
        y = mxfp8_gemm(data, scales, wd, ws, sum(widths), rows=rows, bias=bias)
        return tuple(t.reshape(*x.shape[:-1], w) for t, w in zip(y.split(widths, dim=-1), widths))
    return tuple(p.forward_quantized(data, scales, rows=rows).reshape(*x.shape[:-1], p.out_features)
                 for p in projections)


def convert_linear_to_mxfp8(model, *, enabled=False, chunk_rows=128, check_finite=True):
    """Default-off exact seven-role conversion (mxfp8_linear.py:145-180)."""
    if type(enabled) is not bool or type(check_finite) is not bool:
        raise ValueError("enabled and check_finite must be booleans")
    if not enabled:
        return []
    if model.training:
        raise ValueError("convert an eval model after effective-weight merging")
    targets, seen = [], set()
    parameter_uses = {}
    for _, parameter in model.named_parameters(remove_duplicate=False):
        parameter_uses[id(parameter)] = parameter_uses.get(id(parameter), 0) + 1
    for index, block in enumerate(model.transformer_blocks):
        for role, suffix in SUPPORTED_ROLES.items():
            child = block.get_submodule(suffix)
            if type(child) is not nn.Linear or child.weight.device.type not in ("cpu", "meta"):
                raise ValueError(f"{index}:{role} requires a merged CPU/meta nn.Linear")
            if id(child.weight) in seen or parameter_uses[id(child.weight)] != 1:
                raise ValueError("tied MXFP8 target weights are unsupported")
            seen.add(id(child.weight))
            parent_path, name = suffix.rsplit(".", 1)
            targets.append((index, role, block.get_submodule(parent_path), name, suffix))
    records = []
    for index, role, parent, name, suffix in targets:
        child = getattr(parent, name)
        records.append(dict(block=index, role=role, module=f"transformer_blocks.{index}.{suffix}",
                            in_features=child.in_features, out_features=child.out_features))
        setattr(parent, name, MXFP8Linear(child, chunk_rows=chunk_rows, check_finite=check_finite))
        del child
    return records
