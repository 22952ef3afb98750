"""GPU: vdn_vda_forward_noalloc, the VDA entry point for callers that cannot allocate.

Some callers of this library cannot provide device memory for a workspace or let
the library call cudaMalloc -- a host engine that owns every byte of device
memory through its own pool, or a latency-critical loop that cannot take
cudaMalloc's implicit device synchronisation.  For them the library carries a
fixed 64 MiB scratch array and this entry point uses it instead of a caller
workspace.  This test calls it through the C ABI and checks that two calls in a
row (with different inputs, so stale scratch contents would show) give exactly
the output of the regular workspace entry point, vdn_vda_forward (the two run
the same deterministic kernels, so the results are bit-identical), that the
second call leaves the device's free memory unchanged (it allocates nothing),
and that the size limit sits exactly where the 64 MiB scratch runs out: 20
frames x 10 heads at d = 128 are accepted, 21 x 10 are rejected with a clear
error.

The file is named so that pytest collects it last.
"""
import ctypes as C

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _inputs(f, s, h, d, seed, dev):
    g = torch.Generator(device=dev).manual_seed(seed)
    n = f * s
    q = F.normalize(torch.randn(n, h, d, device=dev, generator=g), dim=-1).bfloat16()
    k = F.normalize(torch.randn(n, h, d, device=dev, generator=g), dim=-1).bfloat16()
    v = torch.randn(n, h, d, device=dev, generator=g).bfloat16()
    beta = torch.sigmoid(torch.randn(n, h, device=dev, generator=g)).bfloat16()
    gate = torch.rand(n, h, d, device=dev, generator=g).bfloat16()
    alpha = torch.exp(-F.softplus(torch.randn(f, h, 1, device=dev, generator=g))).expand(f, h, d).contiguous()
    return q, k, v, beta, gate, alpha


def _call(name, lib_mod, tensors, f, s, h, d, out, bounds, workspace=None):
    q, k, v, beta, gate, alpha = tensors
    w = torch.ones(d, device=q.device)
    buf = (C.c_int32 * (2 * f))(*[x for b in bounds for x in b])
    p = lib_mod.ptr
    args = [p(q), p(k), p(v), q.stride(0), q.stride(1), p(beta), beta.stride(0), beta.stride(1),
            p(gate), gate.stride(0), gate.stride(1), p(alpha), p(w), 1e-6, buf, None, 1, f, s, h, d,
            p(out)]
    if workspace is not None:
        args += [p(workspace), workspace.numel()]
    args.append(lib_mod.stream_of(q.device))
    return getattr(lib_mod.load(), name)(*args)


def _rel_l2(a, b):
    a, b = a.double(), b.double()
    return float((a - b).norm() / b.norm())


@torch.no_grad()
def test_noalloc_matches_workspace_entry_point_twice():
    from vdn_b200 import _lib
    dev = torch.device("cuda", 0)
    f, s, h, d = 7, 96, 3, 128
    bounds = [(t - 1, t + 1) for t in range(f)]
    ws = torch.empty(_lib.load().vdn_vda_workspace_size(f, s, h, d), dtype=torch.uint8, device=dev)
    for call, seed in enumerate((1, 2)):      # two calls in a row, different inputs
        x = _inputs(f, s, h, d, seed, dev)
        want = torch.empty(f * s, h * d, device=dev, dtype=torch.bfloat16)
        got = torch.full_like(want, float("nan"))
        assert _call("vdn_vda_forward", _lib, x, f, s, h, d, want, bounds, ws) == 0
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info(dev)[0]
        rc = _call("vdn_vda_forward_noalloc", _lib, x, f, s, h, d, got, bounds)
        assert rc == 0, _lib.load().vdn_last_error()
        torch.cuda.synchronize()
        if call == 1:                         # the first call may load the scratch's module
            assert torch.cuda.mem_get_info(dev)[0] == free_before
        assert bool(torch.isfinite(got).all())
        assert torch.equal(got, want), _rel_l2(got, want)


@torch.no_grad()
@pytest.mark.parametrize("frames,accepted", [(20, True), (21, False)])
def test_noalloc_size_limit(frames, accepted):
    from vdn_b200 import _lib
    dev = torch.device("cuda", 0)
    f, s, h, d = frames, 8, 10, 128
    need = _lib.load().vdn_vda_workspace_size(f, s, h, d)
    assert (need <= 64 << 20) == accepted
    x = _inputs(f, s, h, d, 3, dev)
    out = torch.empty(f * s, h * d, device=dev, dtype=torch.bfloat16)
    bounds = [(max(t - 1, 0), min(t + 1, f - 1)) for t in range(f)]
    rc = _call("vdn_vda_forward_noalloc", _lib, x, f, s, h, d, out, bounds)
    torch.cuda.synchronize()
    if accepted:
        assert rc == 0, _lib.load().vdn_last_error()
        ws = torch.empty(need, dtype=torch.uint8, device=dev)
        want = torch.empty_like(out)
        assert _call("vdn_vda_forward", _lib, x, f, s, h, d, want, bounds, ws) == 0
        torch.cuda.synchronize()
        assert torch.equal(out, want)
    else:
        assert rc == _lib.VDN_ERR_VALUE
        assert "scratch" in _lib.load().vdn_last_error().decode()


@torch.no_grad()
def test_noalloc_rejects_geometry_beyond_scratch():
    from vdn_b200 import _lib
    dev = torch.device("cuda", 0)
    f, s, h, d = 21, 8, 40, 128               # needs about 236 MiB of scratch
    x = _inputs(f, s, h, d, 3, dev)
    out = torch.empty(f * s, h * d, device=dev, dtype=torch.bfloat16)
    rc = _call("vdn_vda_forward_noalloc", _lib, x, f, s, h, d, out, [(t - 1, t + 1) for t in range(f)])
    assert rc == _lib.VDN_ERR_VALUE
    assert "scratch" in _lib.load().vdn_last_error().decode()
