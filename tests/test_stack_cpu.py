"""CPU: the denoise loop's host logic -- the shard of the packed [text | video] sequence
each Ulysses rank holds, and the Euler update -- with a stand-in for the stack."""
from types import SimpleNamespace

import pytest
import torch

from vdn_b200.stack import denoise, local_rows
from vdn_b200.ulysses import sequence_splits


class _Echo:
    """Stand-in stack: returns its input times two (records the calls)."""

    def __init__(self):
        self.calls = []

    def __call__(self, packed, temb, frames, tokens, runtime=None, text_rows=0):
        self.calls.append((packed.clone(), text_rows, runtime))
        return packed * 2


@pytest.mark.parametrize("L,T,P", [(5, 24, 3), (16, 48, 4), (0, 12, 2), (30, 10, 4)])
def test_shards_cover_the_packed_sequence(L, T, P):
    splits = sequence_splits(L + T, P)
    seen_t, seen_v = [], []
    start = 0
    for r, rows in enumerate(splits):
        rt = SimpleNamespace(world_size=P, local_start=start, local_end=start + rows)
        (ta, tb), (va, vb) = local_rows(L, rt)
        assert (tb - ta) + (vb - va) == rows
        seen_t += list(range(ta, tb))
        seen_v += list(range(va, vb))
        start += rows
    assert seen_t == list(range(L)) and seen_v == list(range(T))


def test_denoise_sharded_matches_whole():
    L, F, S, hd, steps = 6, 3, 4, 8, 2
    T = F * S
    text = torch.randn(steps, L, hd)
    video = torch.randn(T, hd)
    tembs = torch.randn(steps, hd)
    whole = denoise(_Echo(), video.clone(), text, tembs, F, S)
    want = video.clone()
    for _ in range(steps):
        want = want + (-0.5) * (want * 2)
    assert torch.allclose(whole, want)
    splits = sequence_splits(L + T, 3)
    start = 0
    for rows in splits:
        rt = SimpleNamespace(world_size=3, local_start=start, local_end=start + rows,
                             sequence_length=L + T)
        (ta, tb), (va, vb) = local_rows(L, rt)
        echo = _Echo()
        shard = denoise(echo, video[va:vb].clone(), text, tembs, F, S, runtime=rt)
        assert torch.allclose(shard, whole[va:vb])
        packed0, text_rows, got_rt = echo.calls[0]
        assert text_rows == L and got_rt is rt
        assert torch.equal(packed0[:tb - ta], text[0, ta:tb])
        start += rows
    bad = SimpleNamespace(world_size=3, local_start=0, local_end=6, sequence_length=L + T + 1)
    with pytest.raises(ValueError):
        denoise(_Echo(), video[:0].clone(), text, tembs, F, S, runtime=bad)


def test_block_config_layout_arguments():
    from vdn_b200.block import BlockConfig
    assert BlockConfig().plain_window
    assert not BlockConfig(anchor_frames="both").plain_window
    assert not BlockConfig(chunk=5).plain_window
    assert BlockConfig(text_state=1).text_state is True
    for bad in (dict(anchor_frames="corners"), dict(chunk=-1), dict(radius=-1)):
        with pytest.raises(ValueError):
            BlockConfig(**bad)
