"""The attention work list (host code of the forward, through the C ABI
ffwd_b200_attention_items): every (sequence, query head, query tile) is covered
exactly once, items carry the right key-tile counts, and the ordering the
kernel relies on for load balance and L2 reuse holds.  CPU only."""

import collections

import numpy as np
import pytest
from hypothesis import given, settings, strategies as st

from ffwd_b200 import native

LENS = [1, 2, 127, 128, 129, 255, 256, 300, 1000, 2049, 64, 7]


def tiles(L, t):
    return (L + t - 1) // t


def check_tc_cover(lens, heads, kv, hd, causal):
    it = native.attention_items(lens, heads, kv, causal=causal)
    seen = collections.Counter()
    for seq, qt0, h0, qt1, h1, cost in it:
        nq = tiles(lens[seq], 128)
        blocks = [(qt0, h0)] + ([(qt1, h1)] if qt1 >= 0 else [])
        for qt, h in blocks:
            assert 0 <= qt < nq and 0 <= h < heads
            seen[(seq, h, qt)] += 1
        # both blocks read the same keys and values
        assert len({h * kv // heads for _, h in blocks}) == 1
        qmax = max(qt for qt, _ in blocks)
        assert cost == (qmax + 1 if causal else nq)
        if heads != kv:  # grouped heads: two heads of one key/value head, same tile
            assert qt1 < 0 or (qt1 == qt0 and h1 == h0 + 1)
        else:            # one head: adjacent query tiles
            assert qt1 < 0 or (h1 == h0 and qt1 == qt0 + 1)
    want = {(s, h, t) for s, L in enumerate(lens) for h in range(heads)
            for t in range(tiles(L, 128))}
    assert set(seen) == want and max(seen.values()) == 1


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("heads,kv,hd", [(16, 8, 128), (32, 8, 128), (12, 12, 64), (12, 12, 32),
                                         (16, 16, 64)])
def test_tensor_core_items_cover_once(causal, heads, kv, hd):
    check_tc_cover(LENS, heads, kv, hd, causal)


@settings(max_examples=60, deadline=None)
@given(lens=st.lists(st.integers(1, 3000), min_size=1, max_size=24),
       layout=st.sampled_from([(16, 8, 128), (32, 8, 128), (12, 12, 64), (16, 16, 32),
                               (14, 2, 64), (24, 8, 128)]),
       causal=st.booleans())
def test_tensor_core_items_cover_once_random(lens, layout, causal):
    check_tc_cover(lens, *layout, causal)


def test_tensor_core_item_order():
    """Longest sequence first; within a sequence the items of one key/value
    head are contiguous, heaviest query tile first."""
    it = native.attention_items(LENS, 16, 8, causal=True)
    seq_order = [s for i, s in enumerate(it[:, 0]) if i == 0 or s != it[i - 1, 0]]
    assert len(seq_order) == len(set(seq_order))  # each sequence in one run
    lens = [LENS[s] for s in seq_order]
    assert lens == sorted(lens, reverse=True)
    for s in seq_order:
        rows = it[it[:, 0] == s]
        kvh = rows[:, 2] // 2
        runs = [k for i, k in enumerate(kvh) if i == 0 or k != kvh[i - 1]]
        assert len(runs) == len(set(runs))
        for k in runs:
            qts = rows[kvh == k][:, 1]
            assert list(qts) == sorted(qts, reverse=True)


def test_bad_arguments():
    L = native.lib()
    offs = np.array([0, 4], np.int32)
    assert L.ffwd_b200_attention_items(1, 12, 5, offs.ctypes.data, 1, None, 0) == -1
    out = np.zeros((1, 6), np.int32)
    # 16 heads over 8 kv heads, 4 tokens: 8 items do not fit in 1
    assert L.ffwd_b200_attention_items(1, 16, 8, offs.ctypes.data, 1, out.ctypes.data, 1) == -1
