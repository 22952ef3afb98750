"""CPU: the window-softmax launch plan (text rows, anchor frames, frame and chunk
windows) end to end, with the two device calls replaced by CPU stand-ins:

* the cuDNN attention call by an fp32 attention that returns the same layouts
  (token-major bf16 output, fp32 log-sum-exp);
* the vdn_window_merge launch by a restatement of its indexing that reads and
  writes the raw addresses it is given, and first checks that every partial
  row, log-sum-exp, gate and output element it touches lies inside a buffer
  the plan allocated for it.

So the pointer offsets, batch / frame ranges and merge grouping that the GPU
kernel receives are checked here for every layout, against the reference
window softmax (oracle.window, pinned to the reference).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import window as ow
from vdn_b200 import window as win


class _Buffers:
    def __init__(self):
        self.spans = []

    def add(self, t):
        self.spans.append((t.data_ptr(), t.data_ptr() + t.untyped_storage().nbytes()
                           - t.storage_offset() * t.element_size(), t))
        return t

    def check(self, lo, hi, what):
        assert any(a <= lo and hi <= b for a, b, _ in self.spans), f"{what}: [{lo:#x}, {hi:#x}) outside"


def _array(ptr, count, ctype, dtype):
    return np.ctypeslib.as_array((ctype * count).from_address(ptr)).view(dtype)


def _bf16_round(x):
    return torch.from_numpy(np.asarray(x, np.float32)).bfloat16().float().numpy()


@pytest.fixture
def fake_device(monkeypatch):
    bufs = _Buffers()
    calls = []

    def attend(qv, kv, vv, scale):
        q, k, v = qv.float(), kv.float(), vv.float()
        sc = torch.einsum("bhqd,bhkd->bhqk", q, k) * scale
        lse = torch.logsumexp(sc, -1)
        o = torch.einsum("bhqk,bhkd->bhqd", torch.softmax(sc, -1), v).bfloat16()
        o_tm = bufs.add(o.permute(0, 2, 1, 3).contiguous())
        return o_tm.permute(0, 2, 1, 3), bufs.add(lse.contiguous())

    real_flat = win._flat_leg

    def flat_leg(*a, **k):
        leg = real_flat(*a, **k)
        bufs.add(leg[1])
        return leg

    def call(name, n, outs, lses, b0, flo, fhi, F, S, H, d, gate, g_ss, g_sh, out, out_ld, out_hs,
             q, s, stream):
        assert name == "vdn_window_merge" and q is None and s is None
        assert 1 <= n <= win._MAX_PARTIALS
        calls.append(n)
        K = H * d
        parts = []
        for j in range(n):
            assert 0 <= flo[j] <= fhi[j] < F and flo[j] - b0[j] >= 0
            nb = fhi[j] - b0[j] + 1
            po, pl = outs[j], lses[j]
            bufs.check(po, po + nb * S * K * 2, "partial out")
            bufs.check(pl, pl + nb * H * S * 4, "partial lse")
            parts.append((_array(po, nb * S * K, C.c_uint16, np.uint16), _array(pl, nb * H * S, C.c_float,
                                                                               np.float32)))
        gate_p, out_p = gate.value, out.value
        last = (F * S - 1) * out_ld + (H - 1) * out_hs + d
        bufs.check(out_p, out_p + last * 2, "out")
        bufs.check(gate_p, gate_p + ((F * S - 1) * g_ss + (H - 1) * g_sh + 1) * 2, "gate")
        o_arr = _array(out_p, last, C.c_uint16, np.uint16)
        g_arr = _array(gate_p, (F * S - 1) * g_ss + (H - 1) * g_sh + 1, C.c_uint16, np.uint16)
        for r in range(F * S):
            f, sidx = divmod(r, S)
            for h in range(H):
                lse = [(-np.inf if not flo[j] <= f <= fhi[j] else
                        parts[j][1][((f - b0[j]) * H + h) * S + sidx]) for j in range(n)]
                m = max(lse)
                acc, wsum = np.zeros(d, np.float32), 0.0
                for j in range(n):
                    if lse[j] == -np.inf:
                        continue
                    w = np.exp(lse[j] - m)
                    wsum += w
                    row = parts[j][0][((f - b0[j]) * S + sidx) * K + h * d:][:d]
                    acc += w * (row.astype(np.uint32) << 16).view(np.float32)
                val = _bf16_round(acc / wsum)
                gt = (np.uint32(g_arr[r * g_ss + h * g_sh]) << 16).view(np.float32)
                val = _bf16_round(val * gt)
                bits = (val.view(np.uint32) >> 16).astype(np.uint16)
                o_arr[r * out_ld + h * out_hs:][:d] = bits
        return 0

    monkeypatch.setattr(win, "_attend", attend)
    monkeypatch.setattr(win, "_flat_leg", flat_leg)
    monkeypatch.setattr(win._lib, "call", call)
    monkeypatch.setattr(win._lib, "stream_of", lambda dev: None)
    return bufs, calls


CASES = [
    # text rows, frames, tokens, heads, head dim, radius, chunk, anchors
    (0, 6, 4, 2, 8, 1, 0, "none"),
    (3, 6, 4, 2, 8, 1, 0, "both"),
    (2, 7, 3, 2, 8, 1, 2, "columns"),
    (0, 5, 4, 1, 8, 0, 0, "rows"),
    (4, 9, 2, 2, 8, 2, 0, "both"),
    (1, 12, 2, 1, 8, 1, 0, "columns"),
    (2, 5, 3, 2, 8, 0, 2, "both"),
    (0, 4, 3, 2, 8, 3, 0, "none"),
    (5, 1, 4, 2, 8, 1, 0, "both"),
]


@pytest.mark.parametrize("L,f,s,h,d,radius,chunk,anchors", CASES)
def test_plan_matches_reference_window(fake_device, L, f, s, h, d, radius, chunk, anchors):
    bufs, calls = fake_device
    g = torch.Generator().manual_seed(L * 1000 + f * 10 + radius)
    n = L + f * s
    qkv = torch.randn(n, 3, h, d, generator=g).bfloat16()
    q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]                     # strided views, as in the block
    gate = bufs.add(torch.rand(n, h, generator=g).bfloat16())
    out = bufs.add(torch.zeros(n, h, d + 8, dtype=torch.bfloat16))  # head stride > d
    bounds = ow.window_bounds(f, radius, chunk)
    win.window_softmax(q, k, v, gate, f, s, radius, out=out[:, :, :d], bounds=bounds, text_rows=L,
                       anchor_frames=anchors)
    ref = ow.window_attention(q.float(), k.float(), v.float(), f, s, bounds, d ** -0.5, text_rows=L,
                              anchor_frames=anchors)
    ref = (ref.bfloat16().float() * gate.float()[..., None]).bfloat16().float()
    got = out[:, :, :d].float()
    err = float((got - ref).norm() / ref.norm())
    assert err < 6e-3, err
    assert torch.all(out[:, :, d:] == 0)                        # the padding columns untouched
    assert calls and all(c <= win._MAX_PARTIALS for c in calls)


def test_frame_windows_match_oracle_geometry():
    for f in range(1, 9):
        for radius in range(0, 3):
            for chunk in (0, 2, 3):
                bounds = ow.window_bounds(f, radius, chunk)
                for anchors in win.ANCHOR_MODES:
                    assert win.frame_windows(bounds, f, anchors) == ow.frame_keys(bounds, f, anchors)
    with pytest.raises(ValueError):
        win.frame_windows([(2, 1)] * 3, 3)
    with pytest.raises(ValueError):
        win.frame_windows(ow.window_bounds(3, 1), 3, "corners")
