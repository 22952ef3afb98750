"""GPU: the gate GEMM (vdn_gate_gemm) against an fp64 composition of the reference's
eager ops: sigmoid(bf16(x @ w^T + b)) rounded to bf16 on the first n_sig columns,
bf16(x @ w^T + b) after them (reference src/models/attention_gates.py:13-55,
src/models/hybrid_attention.py:108-255).

The kernel sums in fp32, the check in fp64, so the bf16 logit may land one bf16 step
either side of the fp64 one (near a rounding boundary; more for a logit that cancels
below the fp32 summation noise); the sigmoid of a logit one step away can differ by
several bf16 steps of the (smaller) sigmoid value.  So: plain columns
within one bf16 step of the fp64-rounded logit, sigmoid columns between the bf16
sigmoids of the two neighbouring logits, and at most 1 % of all outputs different from
the fp64 composition."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _logits(x, w, b):
    z = x.double() @ w.double().T
    if b is not None:
        z = z + b.double()
    return z.float().bfloat16().float()               # the Linear's bf16 output


def _reference(x, w, b, n_sig):
    z = _logits(x, w, b)
    z[:, :n_sig] = torch.sigmoid(z[:, :n_sig]).bfloat16().float()
    return z


def _check(got, x, w, b, n_sig):
    got = got.float().cpu()
    z = _logits(x, w, b)
    # one bf16 step at z, plus the fp32 summation error of a sum that cancels (2^-16 of
    # the sum of the terms' magnitudes: a small logit can sit below the fp32 noise)
    step = torch.exp2(torch.floor(torch.log2(z.abs().clamp_min(2.0 ** -100))) - 7)
    step = step + 2.0 ** -16 * (x.abs().double() @ w.abs().double().T).float()
    assert bool(((got[:, n_sig:] - z[:, n_sig:]).abs() <= step[:, n_sig:]).all())
    s_lo = torch.sigmoid(z[:, :n_sig] - step[:, :n_sig]).bfloat16().float()
    s_hi = torch.sigmoid(z[:, :n_sig] + step[:, :n_sig]).bfloat16().float()
    assert bool(((got[:, :n_sig] >= s_lo) & (got[:, :n_sig] <= s_hi)).all())
    frac = float((got != _reference(x, w, b, n_sig)).float().mean())
    assert frac < 0.01, frac


@torch.no_grad()
@pytest.mark.parametrize("rows,n,k,n_sig", [(300, 208, 5120, 80), (4096, 5120, 128, 5120), (129, 40, 64, 17),
                                              (1, 256, 192, 0)])
def test_gate_gemm_matches_fp64(cuda, rows, n, k, n_sig):
    from vdn_b200.gates import gate_gemm
    g = torch.Generator().manual_seed(rows + n)
    x = torch.randn(rows, k, generator=g).bfloat16()
    w = (torch.randn(n, k, generator=g) * k ** -0.5).bfloat16()
    b = (torch.randn(n, generator=g) * 0.5).bfloat16()
    y = gate_gemm(x.to(cuda), w.to(cuda), b.to(cuda), n_sig=n_sig)
    torch.cuda.synchronize()
    _check(y, x.float(), w.float(), b.float(), n_sig)


@torch.no_grad()
def test_gate_gemm_strided_views_and_out(cuda):
    """The block's call shapes: the hidden columns of [rows, 2H + r] as a strided view
    (also at an offset the tensor maps cannot take: copied), and `out` views."""
    from vdn_b200.gates import gate_gemm
    g = torch.Generator().manual_seed(5)
    for H in (40, 2):
        g3 = torch.randn(777, 2 * H + 128, generator=g).bfloat16().to(cuda)
        w = (torch.randn(H * 128, 128, generator=g) * 0.1).bfloat16().to(cuda)
        b = torch.randn(H * 128, generator=g).bfloat16().to(cuda)
        hidden = g3[:, 2 * H:]
        y = gate_gemm(hidden, w, b, n_sig=H * 128)
        _check(y, hidden.float().cpu(), w.float().cpu(), b.float().cpu(), H * 128)
        buf = torch.zeros(777, H * 128 + 8, dtype=torch.bfloat16, device=cuda)
        out = buf[:, :H * 128]
        r = gate_gemm(hidden, w, b, n_sig=H * 128, out=out)
        assert r is out and torch.equal(out, y)


def test_gate_gemm_argument_checks(cuda):
    from vdn_b200.gates import gate_gemm
    x = torch.zeros(8, 96, dtype=torch.bfloat16, device=cuda)
    w = torch.zeros(16, 96, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(ValueError, match="multiple of 64"):
        gate_gemm(x, w)
    with pytest.raises(TypeError):
        gate_gemm(x.float(), w.float())
    with pytest.raises(ValueError, match="n_sig"):
        gate_gemm(x[:, :64], w[:, :64], n_sig=17)
