"""numpy restatement of the reference MXFP8 (block-32 E4M3 codes, E8M0 scales).

TEST INFRASTRUCTURE ONLY (see the package docstring).

Follows, in the reference ec-jt/vdn:
  * padded_shape / scale_numel ......... src/models/ops/mxfp8_quant.py:15-23
  * E8M0 exponent rule ................. src/models/ops/mxfp8_quant.py:64-70,
                                         src/models/ops/mxfp8_kernels.py:14-21
  * SWIZZLE_32_4_4 scale addresses ..... src/models/ops/mxfp8_kernels.py:24-27,
                                         src/models/ops/mxfp8_quant.py:31-37
  * quantize_cpu ....................... src/models/ops/mxfp8_quant.py:40-74
  * dequant oracle for the GEMM ........ tests/test_paper_stack_mxfp8_ops.py:14-26
  * finite predicate modes ............. src/models/ops/mxfp8_kernels.py:142-162

The fp32 -> float8_e4m3fn conversion is written out on integer bit patterns
(round to nearest even, sign kept, subnormals included) because numpy has no
fp8 type; it reproduces torch's CPU conversion on every input the quantiser can
produce (|x * 2^-e| <= 448 by construction of the exponent rule).
"""
from __future__ import annotations

import numpy as np


def padded_shape(rows: int, k: int) -> tuple[int, int]:
    if rows < 0 or k <= 0:
        raise ValueError("rows must be nonnegative and K positive")
    return ((rows + 127) // 128 * 128, (k + 127) // 128 * 128)


def scale_numel(rows: int, k: int) -> int:
    rp, kp = padded_shape(rows, k)
    return rp * (kp // 32)


def scale_offsets(rows: int, k_padded: int) -> np.ndarray:
    """Flat byte offset of natural scale [r, c] in the SWIZZLE_32_4_4 layout."""
    r = np.arange(rows, dtype=np.int64)[:, None]
    c = np.arange(k_padded // 32, dtype=np.int64)[None, :]
    tile = (r // 128) * (k_padded // 128) + c // 4
    return tile * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + c % 4


def swizzle(natural: np.ndarray) -> np.ndarray:
    """Natural padded [RP, KP/32] uint8 scales -> flat swizzled bytes."""
    rp, c = natural.shape
    if natural.dtype != np.uint8 or rp % 128 or c % 4:
        raise ValueError("expected uint8 scales padded to 128 rows and 4 columns")
    out = np.zeros(rp * c, dtype=np.uint8)
    out[scale_offsets(rp, c * 32)] = natural
    return out


def unswizzle(flat: np.ndarray, rows: int, k_padded: int) -> np.ndarray:
    return flat[scale_offsets(rows, k_padded)]


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns, round to nearest even (finite inputs)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (b + 0x7FFF + ((b >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 values rounded to bf16 (round to nearest even), as float32.  Uses torch's
    conversion (multithreaded), which equals f32_to_bf16_bits on every finite input."""
    import torch
    t = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))
    return t.to(torch.bfloat16).float().numpy()


def _rne_shift(value: np.ndarray, shift: np.ndarray) -> np.ndarray:
    """Round value / 2**shift to nearest even; value, shift int64, shift >= 1."""
    shift = np.minimum(shift, 62)
    q = value >> shift
    rem = value & ((np.int64(1) << shift) - 1)
    half = np.int64(1) << (shift - 1)
    up = (rem > half) | ((rem == half) & ((q & 1) == 1))
    return q + up.astype(np.int64)


def f32_to_e4m3_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> float8_e4m3fn bytes, round to nearest even, |x| <= 448."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.int64)
    sign = (bits >> 31) & 1
    exp = (bits >> 23) & 0xFF
    man = bits & 0x7FFFFF
    if np.any(exp == 0xFF):
        raise ValueError("nonfinite value reached the E4M3 conversion")
    # Normal E4M3 result (biased exponent >= 1): keep 3 of 23 mantissa bits.
    e8 = exp - 120
    joined = (np.maximum(e8, 0) << 23) | man
    normal = _rne_shift(joined, np.full_like(joined, 20))
    # E4M3 subnormal (units of 2^-9) from the full significand 1.m * 2^(exp-127).
    full = np.where(exp > 0, man | (1 << 23), man)
    eff = np.where(exp > 0, exp, 1)
    sub = _rne_shift(full, 141 - eff)
    code = np.where(e8 >= 1, normal, sub)
    if np.any(code > 0x7E):
        raise ValueError("value outside the E4M3 finite range reached the quantiser")
    return (code | (sign << 7)).astype(np.uint8)


def e4m3_bits_to_f32(codes: np.ndarray) -> np.ndarray:
    c = codes.astype(np.int64)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 7
    val = np.where(e == 0, m / 8.0 * 2.0 ** -6, (1 + m / 8.0) * 2.0 ** (e - 7))
    val = np.where((c & 0x7F) == 0x7F, np.nan, val)
    return (sign * val).astype(np.float32)


def e8m0_rule(amax: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Block exponent e and the exact power-of-two multiplier 2^-e (fp32)."""
    amax = np.ascontiguousarray(amax, dtype=np.float32)
    bits = amax.view(np.int32).astype(np.int64)
    e0 = ((bits >> 23) & 255) - 135
    thr = ((((e0 + 135) << 23) | 0x600000).astype(np.int32)).view(np.float32)
    e = np.maximum(e0 + (amax > thr).astype(np.int64), -127)
    inv = (((127 - e) << 23).astype(np.int32)).view(np.float32)
    return e, inv


def quantize(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """[rows, K] float32 (values of a bf16/fp16/fp32 matrix) -> padded codes, scales.

    Returns uint8 [RP, KP] codes and flat uint8 [RP*KP/32] swizzled E8M0 bytes;
    the padding holds exact zeros (code 0, scale byte 0).
    """
    x = np.asarray(x, dtype=np.float32)
    if x.ndim != 2:
        raise ValueError("expected a 2D matrix")
    if not np.isfinite(x).all():
        raise ValueError("nonfinite MXFP8 input")
    r, k = x.shape
    rp, kp = padded_shape(r, k)
    values = np.zeros((rp, kp), dtype=np.float32)
    values[:r, :k] = x
    blocks = values.reshape(rp, kp // 32, 32)
    amax = np.abs(blocks).max(-1)
    e, inv = e8m0_rule(amax)
    scaled = (blocks * inv[..., None]).reshape(rp, kp)
    codes = f32_to_e4m3_bits(scaled)
    natural = (e + 127).astype(np.uint8)
    return codes, swizzle(natural)


def dequantize(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    rp, kp = codes.shape
    natural = unswizzle(scales, rp, kp).astype(np.float64)
    vals = e4m3_bits_to_f32(codes).astype(np.float64).reshape(rp, kp // 32, 32)
    return (vals * np.exp2(natural - 127)[..., None]).reshape(rp, kp)


def qdq_torch(x):
    """MXFP8 quantise-then-dequantise of a [rows, K] CPU tensor: the fp32 values the GEMM
    multiplies (cropped to [rows, K]).  The same rule as quantize() (quantize_cpu,
    src/models/ops/mxfp8_quant.py:40-74) in multithreaded torch CPU ops, with torch's
    float8_e4m3fn conversion (round to nearest even) in place of the bit-pattern
    restatement; pinned bit-exact against dequantize(quantize(x)) by the CPU tests.
    For the full-size checks, where the numpy path takes minutes."""
    import torch
    r, k = x.shape
    kp = (k + 127) // 128 * 128
    v = torch.zeros(r, kp, dtype=torch.float32)
    v[:, :k] = x.float()
    if not bool(torch.isfinite(v).all()):
        raise ValueError("nonfinite MXFP8 input")
    blocks = v.view(r, kp // 32, 32)
    amax = blocks.abs().amax(-1)
    bits = amax.view(torch.int32)
    e0 = ((bits >> 23) & 255) - 135
    thr = (((e0 + 135) << 23) | 0x600000).view(torch.float32)
    e = (e0 + (amax > thr).to(torch.int32)).clamp_min(-127)
    inv = ((127 - e) << 23).view(torch.float32)
    codes = (blocks * inv[..., None]).to(torch.float8_e4m3fn)
    out = codes.to(torch.float64) * torch.pow(2.0, e.to(torch.float64))[..., None]
    return out.view(r, kp)[:, :k].to(torch.float32)


def mxfp8_gemm(xq, xs, wq, ws, rows, n, bias=None) -> np.ndarray:
    """Dequantised fp64 GEMM oracle, cropped to [rows, n], rounded to bf16 (+bias)."""
    y = dequantize(xq, xs) @ dequantize(wq, ws).T
    y = round_bf16(y[:rows, :n].astype(np.float32))
    if bias is not None:
        y = round_bf16(y + round_bf16(bias))
    return y


def finite_parts(x: np.ndarray, mode: int = 0, block: int = 4096) -> np.ndarray:
    """Per-4096-element finite predicate: floats, E4M3 codes or E8M0 bytes."""
    flat = np.ravel(x)
    if mode == 1:
        good = (flat.astype(np.uint8) & 127) != 127
    elif mode == 2:
        good = flat.astype(np.uint8) != 255
    else:
        good = np.isfinite(flat.astype(np.float32))
    n = (flat.size + block - 1) // block
    pad = np.ones(n * block, dtype=bool)
    pad[:flat.size] = good
    return pad.reshape(n, block).all(1)
