"""paper_delta_factors on the B200 factor kernel.

Same contract as ec-jt/vdn src/models/linear_attention/paper_factor.py:133-186:
returns (diag(alpha) @ inv(I + A), B @ inv(I + A)) for contiguous fp32 CUDA
tensors of shape [..., d, d] (d = 128, also 64 here), alpha [..., d] or None.
Invalid metadata raises TypeError / ValueError before any launch; unsupported
hardware or a failed launch raises RuntimeError.  No input is mutated; outputs
are fresh allocations; misaligned contiguous inputs are cloned to 16 bytes.
"""
from __future__ import annotations

import torch

from . import _lib

__all__ = ["paper_delta_factors"]


def _check_tensor(t, name: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.dtype != torch.float32:
        raise TypeError(f"{name} must have dtype float32, got {t.dtype}")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.layout != torch.strided or not t.is_contiguous():
        raise ValueError(f"{name} must have contiguous strided storage")
    if t.requires_grad:
        raise ValueError(f"{name} requires_grad is unsupported by this inference-only kernel")
    if t.is_conj() or t.is_neg():
        raise ValueError(f"{name} must not have unresolved conjugate/negative view bits")


def _aligned(t: torch.Tensor) -> torch.Tensor:
    return t if t.data_ptr() % 16 == 0 else t.clone()


def paper_delta_factors(A, B, alpha=None):
    """Return ``(diag(alpha) @ inv(I + A), B @ inv(I + A))`` for SPD I + A."""
    _check_tensor(A, "A")
    _check_tensor(B, "B")
    if A.ndim < 2 or A.shape[-1] != A.shape[-2] or A.shape[-1] not in (64, 128):
        raise ValueError("A must have shape [..., d, d] with d in (64, 128)")
    d = A.shape[-1]
    if B.shape != A.shape:
        raise ValueError("B shape must exactly equal A shape")
    if B.device != A.device:
        raise ValueError("A and B must be on the same CUDA device")
    if alpha is not None:
        _check_tensor(alpha, "alpha")
        if alpha.shape != A.shape[:-1]:
            raise ValueError("alpha must have exact shape [..., d] matching A")
        if alpha.device != A.device:
            raise ValueError("alpha must be on the same CUDA device as A")
    _lib.require_device(A, "A")
    T = torch.empty_like(A)
    J = torch.empty_like(B)
    if A.numel() == 0:
        return T, J
    n = A.numel() // (d * d)
    with torch.cuda.device(A.device):
        a, b = _aligned(A), _aligned(B)
        al = None if alpha is None else _aligned(alpha)
        _lib.call("vdn_delta_factors", _lib.ptr(a), _lib.ptr(b), _lib.ptr(al), n, d,
                  _lib.ptr(T), _lib.ptr(J), _lib.stream_of(A.device))
    return T, J
