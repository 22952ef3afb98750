"""MXFP8 storage envelope and shard repacking (CPU).

Follows the reference's serialization gate (scripts/benchmark_rtx5090_real_mxfp8.py:34-68)
and its tensor-parallel repack (src/inference/utils/tensor_parallel.py:20-62):
records round-trip bit for bit, malformed records are rejected, and a repacked
shard equals the quantisation of the selected floating sub-matrix.
"""
import pytest
import torch

from vdn_b200.mxfp8_format import (FORMAT, load_prepared, pack_prepared, save_prepared,
                                   shard_prepared, unpack_prepared, unswizzle_scales)
from vdn_b200.mxfp8_quant import quantize_cpu, swizzle_scales


def _weight(n, k, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(n, k, generator=g) * 0.02).bfloat16()


def test_envelope_round_trip(tmp_path):
    q, s = quantize_cpu(_weight(200, 300))
    rec = pack_prepared(q, s)
    assert rec["format"] == FORMAT and rec["q"].data_ptr() != q.data_ptr()
    q2, s2 = unpack_prepared(rec)
    assert torch.equal(q2, q) and torch.equal(s2, s)
    digest = save_prepared(tmp_path / "w.pt", q, s)
    assert len(digest) == 64
    q3, s3 = load_prepared(tmp_path / "w.pt")
    assert torch.equal(q3, q) and torch.equal(s3, s)
    with pytest.raises(FileExistsError):
        save_prepared(tmp_path / "w.pt", q, s)
    # float8 views are accepted and stored as bytes
    rec8 = pack_prepared(q.view(torch.float8_e4m3fn), s)
    assert rec8["q"].dtype == torch.uint8


@pytest.mark.parametrize("mutate", ["format", "qdtype", "sdtype", "shape", "bytes"])
def test_envelope_rejects_malformed(mutate):
    q, s = quantize_cpu(_weight(128, 128))
    rec = pack_prepared(q, s)
    if mutate == "format":
        rec["format"] = "mxfp8-v0"
    elif mutate == "qdtype":
        rec["q_dtype"] = "torch.uint8"
    elif mutate == "sdtype":
        rec["scale_dtype"] = "torch.uint8"
    elif mutate == "shape":
        rec["scale"] = rec["scale"][:-1]
    else:
        rec["q"] = rec["q"].float()
    with pytest.raises(ValueError):
        unpack_prepared(rec)


def test_unswizzle_inverts_swizzle():
    g = torch.Generator().manual_seed(4)
    natural = torch.randint(0, 255, (256, 12), generator=g, dtype=torch.uint8)
    assert torch.equal(unswizzle_scales(swizzle_scales(natural), 256, 384), natural)


@pytest.mark.parametrize("rows,cols", [(None, (64, 300)), ([5, 0, 199, 77, 3], None),
                                       (list(range(10, 150, 3)), (32, 256)), ([7], (288, 300))])
def test_shard_equals_quantised_submatrix(rows, cols):
    n, k = 200, 300
    w = _weight(n, k, seed=1)
    q, s = quantize_cpu(w)
    qs, ss = shard_prepared(q, s, n, k, rows=rows, columns=cols)
    r = list(range(n)) if rows is None else rows
    a, b = (0, k) if cols is None else cols
    want_q, want_s = quantize_cpu(w[r][:, a:b].contiguous())
    assert torch.equal(qs, want_q) and torch.equal(ss, want_s)


def test_shard_rejects_unaligned_k():
    q, s = quantize_cpu(_weight(64, 256))
    with pytest.raises(ValueError):
        shard_prepared(q, s, 64, 256, columns=(16, 128))
    with pytest.raises(ValueError):
        shard_prepared(q, s, 64, 256, rows=[0, 0])
