"""The hybrid block's gate projections on the tcgen05 bf16 GEMM (vdn_gate_gemm).

    gate_gemm(x, w, bias, n_sig)  ->  act(bf16(x @ w.T + bias))

with act = sigmoid (rounded to bf16) on the first n_sig output columns: an eager bf16
nn.Linear followed by torch.sigmoid, as the reference computes the softmax gate, the
beta projection (src/models/hybrid_attention.py:108-255) and the linear branch's
OutputGate (src/models/attention_gates.py:13-55: down, then sigmoid(up(.))).
"""
from __future__ import annotations

import torch

from . import _lib
from .mxfp8_linear import _status

__all__ = ["gate_gemm"]


def _tma_ok(t: torch.Tensor) -> bool:
    return (t.stride(-1) == 1 and t.stride(0) % 8 == 0 and t.stride(0) >= t.shape[1]
            and t.data_ptr() % 16 == 0)


def gate_gemm(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None, n_sig: int = 0,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """bf16 [rows, n] = act(bf16(x [rows, k] @ w [n, k]^T + bias [n])), sigmoid on columns
    < n_sig.  k must be a multiple of 64; strided row views are accepted (copied when
    their layout does not suit the tensor maps)."""
    if x.dim() != 2 or w.dim() != 2 or x.shape[1] != w.shape[1]:
        raise ValueError("x must be [rows, k] and w [n, k]")
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or not x.is_cuda or w.device != x.device:
        raise TypeError("x and w must be bf16 CUDA tensors on one device")
    rows, k = x.shape
    n = w.shape[0]
    if k % 64:
        raise ValueError(f"k must be a multiple of 64, got {k}")
    if not 0 <= n_sig <= n:
        raise ValueError("n_sig must lie in [0, n]")
    _lib.require_device(x)
    if not _tma_ok(x):
        x = x.contiguous()
    if not _tma_ok(w):
        w = w.contiguous()
    if bias is not None:
        if bias.shape != (n,) or bias.dtype != torch.bfloat16:
            raise ValueError("bias must be bf16 [n]")
        bias = bias.contiguous()
    target = out
    if out is None or out.shape != (rows, n) or out.dtype != torch.bfloat16 or not _tma_ok(out):
        # rows padded to a multiple of 8 elements (the store map's 16-byte row pitch)
        target = torch.empty(rows, (n + 7) // 8 * 8, device=x.device, dtype=torch.bfloat16)[:, :n]
    _lib.call("vdn_gate_gemm", _lib.ptr(x), x.stride(0), _lib.ptr(w), w.stride(0), _lib.ptr(bias), rows, n, k,
              n_sig, _lib.ptr(target), target.stride(0), _lib.ptr(_status(x.device)), _lib.stream_of(x.device))
    if out is not None and target is not out:
        out.copy_(target)
        return out
    return target
