"""MXFP8 storage / wire format and weight-shard repacking.

Byte envelope for prepared MXFP8 operands (E4M3 codes as uint8, E8M0 scales as
uint8 in the SWIZZLE_32_4_4 order the GEMM consumes), with the reference's
format tag so records interchange with it (scripts/benchmark_rtx5090_real_mxfp8.py:34-68:
FORMAT, pack_prepared, unpack_prepared), and the scale un-swizzle / shard repack
of src/inference/utils/tensor_parallel.py:20-62 (unswizzle_scales, the MXFP8 branch
of shard_linear): selecting output rows and a 32-aligned K range of a prepared
weight without going back to floating point.
"""
from __future__ import annotations

import hashlib
from pathlib import Path

import torch

from .mxfp8_quant import padded_shape, swizzle_scales

__all__ = ["FORMAT", "pack_prepared", "unpack_prepared", "unswizzle_scales", "shard_prepared",
           "save_prepared", "load_prepared"]

FORMAT = "mxfp8-e4m3fn-e8m0-block32-swizzle32_4_4-v1"
_Q_DTYPE = "torch.float8_e4m3fn"
_S_DTYPE = "torch.float8_e8m0fnu"


def _as_bytes(t: torch.Tensor, name: str) -> torch.Tensor:
    if t.dtype in (torch.uint8,):
        return t
    if t.dtype == torch.float8_e4m3fn or str(t.dtype) == _S_DTYPE:
        return t.view(torch.uint8)
    raise ValueError(f"{name} must be uint8 bytes or the matching float8 dtype, got {t.dtype}")


def pack_prepared(q: torch.Tensor, scale: torch.Tensor) -> dict:
    """Independent CPU byte copies of codes [RP, KP] and swizzled scales [RP*KP/32]."""
    if q.ndim != 2 or q.shape[0] % 128 or q.shape[1] % 128:
        raise ValueError("codes must be a padded [RP, KP] matrix (multiples of 128)")
    qb, sb = _as_bytes(q, "codes"), _as_bytes(scale, "scales")
    if sb.numel() != q.shape[0] * q.shape[1] // 32:
        raise ValueError("scale count does not match the padded codes")
    return {"format": FORMAT, "q": qb.detach().cpu().clone().contiguous(),
            "scale": sb.detach().reshape(-1).cpu().clone().contiguous(),
            "q_dtype": _Q_DTYPE, "scale_dtype": _S_DTYPE}


def unpack_prepared(record: dict) -> tuple[torch.Tensor, torch.Tensor]:
    """(codes uint8 [RP, KP], scales uint8 [RP*KP/32]) after validating the envelope."""
    if record.get("format") != FORMAT:
        raise ValueError("invalid MXFP8 serialization format")
    q, s = record.get("q"), record.get("scale")
    if not isinstance(q, torch.Tensor) or not isinstance(s, torch.Tensor) or \
            q.dtype != torch.uint8 or s.dtype != torch.uint8:
        raise ValueError("invalid MXFP8 serialization format")
    if record.get("q_dtype") != _Q_DTYPE or record.get("scale_dtype") != _S_DTYPE:
        raise ValueError("invalid MXFP8 dtype metadata")
    if q.ndim != 2 or q.shape[0] % 128 or q.shape[1] % 128 or s.numel() != q.numel() // 32:
        raise ValueError("invalid MXFP8 record shape")
    return q, s


def unswizzle_scales(scales: torch.Tensor, rows: int, k: int) -> torch.Tensor:
    """Natural [RP, KP/32] scales from the SWIZZLE_32_4_4 order (tensor_parallel.py:20-26)."""
    rp, kp = padded_shape(rows, k)
    if scales.numel() != rp * kp // 32:
        raise ValueError("scale count does not match the padded shape")
    return (scales.reshape(-1, 32, 4, 4).transpose(1, 2)
            .reshape(rp // 128, kp // 128, 128, 4).permute(0, 2, 1, 3)
            .reshape(rp, kp // 32).contiguous())


def shard_prepared(q: torch.Tensor, scale: torch.Tensor, n: int, k: int, *, rows=None, columns=None):
    """Repack selected output rows and a 32-aligned K range [start, end) of a prepared
    [n, k] weight into independent padded storage (tensor_parallel.py:45-56).

    The result equals quantising the selected floating sub-matrix: MXFP8 blocks are
    per row and per 32 K, so selection commutes with quantisation.
    """
    rows = list(range(n)) if rows is None else list(rows)
    start, end = (0, k) if columns is None else columns
    if not rows or len(set(rows)) != len(rows) or min(rows) < 0 or max(rows) >= n:
        raise ValueError("invalid shard rows")
    if not 0 <= start < end <= k:
        raise ValueError("invalid shard columns")
    if start % 32 or (end % 32 and end != k):
        raise ValueError("MXFP8 K cuts must be block32 aligned")
    qb, sb = _as_bytes(q, "codes"), _as_bytes(scale, "scales")
    idx = torch.tensor(rows, device=qb.device, dtype=torch.long)
    width = end - start
    rp, kp = padded_shape(len(rows), width)
    data = torch.zeros((rp, kp), device=qb.device, dtype=torch.uint8)
    data[: len(rows), :width] = qb.index_select(0, idx)[:, start:end]
    natural = unswizzle_scales(sb.reshape(-1), n, k)
    scales = torch.zeros((rp, kp // 32), device=qb.device, dtype=torch.uint8)
    nb = (width + 31) // 32
    scales[: len(rows), :nb] = natural.index_select(0, idx)[:, start // 32:start // 32 + nb]
    return data, swizzle_scales(scales)


def save_prepared(path, q: torch.Tensor, scale: torch.Tensor) -> str:
    """Write the envelope with torch.save (exclusive create); returns the file's sha256."""
    path = Path(path)
    with path.open("xb") as f:
        torch.save(pack_prepared(q, scale), f)
    digest = hashlib.sha256()
    with path.open("rb") as f:
        for chunk in iter(lambda: f.read(8 << 20), b""):
            digest.update(chunk)
    return digest.hexdigest()


def load_prepared(path) -> tuple[torch.Tensor, torch.Tensor]:
    return unpack_prepared(torch.load(Path(path), map_location="cpu", weights_only=True))
