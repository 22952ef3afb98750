"""Block-32 E4M3/E8M0 preparation: the reference's quantiser API on B200 kernels.

Mirrors ec-jt/vdn src/models/ops/mxfp8_quant.py (padded_shape, scale_numel,
require_finite, swizzle_scales, quantize_cpu, quantize_activation) with the same
names, argument meaning and errors.  quantize_cpu runs the library's native
multithreaded host quantiser; quantize_activation runs the sm_100a kernel, with
the finite check fused into the quantising pass.  Codes and scales are
bit-identical to the reference rule.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib


def padded_shape(rows: int, k: int) -> tuple[int, int]:
    """Rows and K rounded up to multiples of 128 (mxfp8_quant.py:15-18)."""
    if rows < 0 or k <= 0:
        raise ValueError("rows must be nonnegative and K positive")
    return ((rows + 127) // 128 * 128, (k + 127) // 128 * 128)


def scale_numel(rows: int, k: int) -> int:
    rp, kp = padded_shape(rows, k)
    return rp * (kp // 32)


def require_finite(x: torch.Tensor, name: str) -> None:
    if not bool(torch.isfinite(x).all()):
        raise ValueError(f"nonfinite MXFP8 {name}")


def swizzle_scales(scales: torch.Tensor) -> torch.Tensor:
    """Natural padded [rows, K/32] bytes to flat SWIZZLE_32_4_4 bytes (mxfp8_quant.py:31-37)."""
    r, c = scales.shape
    if scales.dtype != torch.uint8 or r % 128 or c % 4:
        raise ValueError("expected uint8 scales padded to 128 rows and 4 columns")
    return (scales.reshape(r // 128, 128, c // 4, 4).permute(0, 2, 1, 3)
            .reshape(-1, 4, 32, 4).transpose(1, 2).reshape(-1).contiguous())


def quantize_cpu(x: torch.Tensor, *, chunk_rows: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Quantise one CPU (or meta) weight matrix; same contract as mxfp8_quant.py:40-74.

    The native host quantiser writes the padded codes and swizzled scales
    directly (no fp32 copy of the matrix).  `chunk_rows` is validated for API
    compatibility; the native routine bounds its temporaries by itself.
    """
    if x.ndim != 2 or x.dtype not in (torch.bfloat16, torch.float16, torch.float32):
        raise ValueError("expected a floating 2D weight")
    if x.device.type not in ("cpu", "meta"):
        raise ValueError("weights must be converted on CPU before distribution")
    if type(chunk_rows) is not int or chunk_rows <= 0:
        raise ValueError("chunk_rows must be a positive integer")
    r, k = x.shape
    rp, kp = padded_shape(r, k)
    data = torch.zeros((rp, kp), dtype=torch.uint8, device=x.device)
    scales = torch.zeros(rp * (kp // 32), dtype=torch.uint8, device=x.device)
    if x.is_meta or r == 0:
        return data, scales
    src = x.detach()
    if src.stride(-1) != 1:
        src = src.contiguous()
    _lib.call("vdn_mxfp8_quantize_host", _lib.ptr(src), _lib.dtype_code(src.dtype), r, k,
              src.stride(0), _lib.ptr(data), _lib.ptr(scales), torch.get_num_threads())
    return data, scales


def _nonfinite_counter(device) -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device)


def quantize_activation(x: torch.Tensor, *, check_finite: bool = True):
    """Fused pad + block-32 quantisation + swizzle of a CUDA bf16 [rows, K] activation.

    Same contract as mxfp8_quant.py:77-90: padded contiguous uint8 codes and
    flat uint8 scales; non-finite input raises ValueError("nonfinite MXFP8
    activation") when check_finite (one host read of a device counter that the
    quantising pass itself fills).
    """
    if x.ndim != 2 or x.dtype != torch.bfloat16 or x.device.type != "cuda":
        raise ValueError("expected CUDA BF16 [rows,K] activation")
    if x.stride(-1) != 1:
        raise ValueError("activation K dimension must be contiguous")
    return launch_quantize(x, check_finite=check_finite)


def launch_quantize(x: torch.Tensor, *, check_finite: bool = False, counter=None):
    """Device quantiser without the input checks of quantize_activation."""
    _lib.require_device(x, "activation")
    r, k = x.shape
    rp, kp = padded_shape(r, k)
    q = torch.empty((rp, kp), dtype=torch.uint8, device=x.device)
    s = torch.empty(scale_numel(r, k), dtype=torch.uint8, device=x.device)
    bad = counter if counter is not None else (_nonfinite_counter(x.device) if check_finite else None)
    _lib.call("vdn_mxfp8_quantize", _lib.ptr(x), r, k, x.stride(0) if r else k, _lib.ptr(q),
              _lib.ptr(s), _lib.ptr(bad), _lib.stream_of(x.device))
    if check_finite and counter is None and int(bad.item()):
        raise ValueError("nonfinite MXFP8 activation")
    return q, s
