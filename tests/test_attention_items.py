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
    for seq, qt0, h0, qt1, h1, cost, nseq in it:
        assert nseq == 0
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


def check_window_cover(lens, heads, kv, causal):
    """The 16-bit plans' list: sequences of 1..128 rows that are neighbours in
    the packed layout share window items; every (head, row) of every sequence
    is covered exactly once; windows come after the single-sequence items."""
    rep = heads // kv
    offs = np.concatenate([[0], np.cumsum(lens)])
    it = native.attention_items(lens, heads, kv, causal=causal, windows=True)
    rows = collections.Counter()
    seen_window = False
    cap = 128 if rep >= 2 else 256
    for seq, qt0, h0, qt1, h1, cost, nseq in it:
        blocks = [(qt0, h0)] + ([(qt1, h1)] if qt1 >= 0 else [])
        assert len({h * kv // heads for _, h in blocks}) == 1
        if nseq == 0:
            assert not seen_window and lens[seq] > 128
            base, L = offs[seq], lens[seq]
            nq = tiles(L, 128)
            assert cost == (max(q for q, _ in blocks) + 1 if causal else nq)
        else:
            seen_window = True
            members = list(range(seq, seq + nseq))
            assert all(1 <= lens[m] <= 128 for m in members)
            base, L = offs[seq], offs[seq + nseq] - offs[seq]
            assert L <= cap
            assert cost == (1 if rep >= 2 else tiles(L, 128))
            if rep >= 2:
                assert qt0 == 0 and (qt1 < 0 or (qt1 == 0 and h1 == h0 + 1))
            else:
                assert qt0 == 0 and (qt1 == 1 and h1 == h0) == (L > 128)
        for qt, h in blocks:
            for r in range(base + qt * 128, base + min(qt * 128 + 128, L)):
                rows[(h, r)] += 1
    want = {(h, r) for h in range(heads) for r in range(int(offs[-1]))}
    assert set(rows) == want and max(rows.values()) == 1
    # a run of short neighbours is cut only where the next one does not fit
    win = [(s, n) for s, *_, n in it if n > 0]
    starts = sorted({s for s, _ in win})
    for s in starts:
        n = dict(win)[s]
        e = s + n
        if e < len(lens) and 1 <= lens[e] <= 128:
            assert offs[e + 1] - offs[s] > cap


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("heads,kv", [(16, 8), (32, 8), (12, 12), (14, 2)])
def test_window_items_cover_once(causal, heads, kv):
    check_window_cover(LENS + [30, 40, 50, 128, 1, 100, 100, 3000, 60], heads, kv, causal)


@settings(max_examples=60, deadline=None)
@given(lens=st.lists(st.one_of(st.integers(1, 140), st.integers(1, 3000)), min_size=1,
                     max_size=40),
       layout=st.sampled_from([(16, 8), (32, 8), (12, 12), (16, 16), (14, 2)]),
       causal=st.booleans())
def test_window_items_cover_once_random(lens, layout, causal):
    check_window_cover(lens, *layout, causal)


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
    assert L.ffwd_b200_attention_items(1, 0, 12, 5, offs.ctypes.data, 1, None, 0) == -1
    out = np.zeros((1, 7), np.int32)
    # 16 heads over 8 kv heads, 4 tokens: 8 items do not fit in 1
    assert L.ffwd_b200_attention_items(1, 0, 16, 8, offs.ctypes.data, 1, out.ctypes.data, 1) == -1
    assert L.ffwd_b200_attention_items(1, 1, 16, 8, offs.ctypes.data, 1, out.ctypes.data, 1) == -1
