"""GPU: the gate GEMM (vdn_gate_gemm) against an fp64 composition of the reference's
eager ops: sigmoid(bf16(x @ w^T + b)) rounded to bf16 on the first n_sig columns,
bf16(x @ w^T + b) after them (reference src/models/attention_gates.py:13-55,
src/models/hybrid_attention.py:108-255).  fp32 accumulation in a different order
from the fp64 sum can move a value across a bf16 rounding boundary, so the bar is
one bf16 ulp on at most 1 % of the outputs (no other difference)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _reference(x, w, b, n_sig):
    z = x.double() @ w.double().T
    if b is not None:
        z = z + b.double()
    z = z.float().bfloat16().float()                 # the Linear's bf16 output
    z[:, :n_sig] = torch.sigmoid(z[:, :n_sig]).bfloat16().float()
    return z


def _check(got, want):
    got = got.float().cpu()
    diff = (got - want).abs()
    ulp = want.abs().clamp_min(2 ** -126) * 2 ** -7   # one bf16 ulp upper bound
    assert bool((diff <= ulp).all()), float(diff.max())
    frac = float((diff > 0).float().mean())
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
    _check(y, _reference(x.float(), w.float(), b.float(), n_sig))


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
        _check(y, _reference(hidden.float().cpu(), w.float().cpu(), b.float().cpu(), H * 128))
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
