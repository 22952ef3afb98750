"""CPU: the operand-plane layout of the d = 128 factor stage (vdn_vda_factor_inverse).

A numpy encoder written from the layout's definition (three bf16 parts, each two
64-column halves of 128 rows x 128 bytes, 16-byte chunk c of row r stored at chunk
c ^ (r % 8)) and the decoder the GPU tests use (split_inverse_values) must be
inverse to each other, and the three-part split must be exact for fp32 values."""
import numpy as np
import torch

from oracle import mxfp8 as omx
from vdn_b200.linear_attention import SPLIT_INVERSE_BYTES, split_inverse_values


def _encode(x):
    """fp32 [128, 128] -> uint8 [98304] in the factor kernel's plane layout."""
    parts, rest = [], x.astype(np.float32)
    for _ in range(3):
        bits = omx.f32_to_bf16_bits(rest)
        val = omx.bf16_to_f32(bits)
        parts.append(bits)
        rest = (rest - val).astype(np.float32)
    assert not rest.any()                              # three parts are exact
    out = np.zeros(SPLIT_INVERSE_BYTES, np.uint8)
    for p, bits in enumerate(parts):
        raw = bits.view(np.uint8).reshape(128, 16, 16)  # row, logical 16-byte chunk, bytes
        for r in range(128):
            for c in range(16):
                kh, cc = c >> 3, c & 7
                off = p * 32768 + kh * 16384 + r * 128 + ((cc ^ (r & 7)) << 4)
                out[off:off + 16] = raw[r, c]
    return out


def test_split_planes_round_trip():
    g = np.random.default_rng(3)
    x = (g.standard_normal((2, 128, 128)) * np.exp2(g.integers(-20, 20, (2, 128, 128)))).astype(np.float32)
    planes = torch.from_numpy(np.stack([_encode(m) for m in x]))
    got = split_inverse_values(planes).numpy()
    assert np.array_equal(got.view(np.uint32), x.view(np.uint32))


def test_third_part_is_the_residual_itself():
    """The kernels store the third part without rounding it: what the first two
    round-to-nearest bf16 parts leave has at most 8 significant bits, so it is a bf16
    value already, for every |x| >= 2^-100 (below ~2^-103 the residual is an fp32
    denormal, and the third part keeps only its upper half: an error under 2^-133)."""
    g = np.random.default_rng(11)
    x = (g.standard_normal(2_000_000) * np.exp2(g.integers(-100, 100, 2_000_000))).astype(np.float32)
    x = x[np.abs(x) >= np.float32(2.0 ** -100)]
    rest = x.copy()
    for _ in range(2):
        rest = (rest - omx.bf16_to_f32(omx.f32_to_bf16_bits(rest))).astype(np.float32)
    assert not (rest.view(np.uint32) & 0xFFFF).any()


def test_silu_input_clamp_on_bf16_patterns():
    """The SiLU transforms raise inputs below -43.5 to -43.5 with one unsigned 16-bit min
    of each packed bf16 against 0xC22E: over all 65536 patterns that is the float clamp
    for every non-NaN value (-inf included), and positive NaNs pass through."""
    bits = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    clamped = np.minimum(bits, np.uint16(0xC22E))
    x = omx.bf16_to_f32(bits)
    y = omx.bf16_to_f32(clamped)
    assert omx.bf16_to_f32(np.array([0xC22E], np.uint16))[0] == -43.5
    ok = ~np.isnan(x)
    want = np.where(x[ok] < -43.5, np.float32(-43.5), x[ok])
    assert np.array_equal(y[ok], want)
    pos_nan = np.isnan(x) & (bits < 0x8000)
    assert np.isnan(y[pos_nan]).all()
