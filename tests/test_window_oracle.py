"""CPU: the window-softmax oracle (global text rows, frame / chunk-aligned windows,
anchor frames) against the reference's own window_softmax_reference run on CPU
(tests/golden/window_golden.npz), and the window geometry helpers."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import window as ow

GOLDEN = Path(__file__).resolve().parent / "golden" / "window_golden.npz"


def _cases():
    z = np.load(GOLDEN)
    names = sorted({k.rsplit("_", 1)[0] for k in z.files if k.endswith("_geom")})
    return z, names


@pytest.mark.parametrize("name", _cases()[1])
def test_oracle_matches_reference_window_softmax(name):
    z = np.load(GOLDEN)
    L, f, s, h, d, radius, chunk = (int(x) for x in z[f"{name}_geom"])
    bounds = ow.window_bounds(f, radius, chunk)
    assert [tuple(b) for b in z[f"{name}_bounds"].tolist()] == bounds
    q, k, v = (torch.from_numpy(z[f"{name}_{t}"]) for t in "qkv")
    got = ow.window_attention(q, k, v, f, s, bounds, d ** -0.5, text_rows=L,
                              anchor_frames=str(z[f"{name}_anchors"]))
    np.testing.assert_allclose(got.numpy(), z[f"{name}_out"], rtol=1e-5, atol=1e-6)


def test_frame_keys_geometry():
    f = 6
    keys = ow.frame_keys(ow.window_bounds(f, 1), f, "both")
    assert keys[0] == (0, 5, []) and keys[5] == (0, 5, [])       # anchor rows: dense
    assert keys[1] == (0, 2, [5]) and keys[3] == (2, 4, [0, 5])   # anchor columns, no repeats
    keys = ow.frame_keys(ow.window_bounds(7, 1, chunk=2), 7, "none")
    assert keys[2] == keys[3] == (0, 5, []) and keys[6] == (4, 6, [])
    assert ow.full_cover(ow.window_bounds(3, 2), 3) and not ow.full_cover(ow.window_bounds(4, 1), 4)
    with pytest.raises(ValueError):
        ow.frame_keys(ow.window_bounds(3, 1), 3, "corners")
