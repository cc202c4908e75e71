"""The stream decode's cost-aware split of the tile stream over its warps,
restated in Python (CPU).

csrc/decode_stream.cu (stream_split / stream_split_start /
stream_split_warp_of): with F(g) = g + cost * u(g), u(g) the index of the unit
holding tile g (KHG units per sequence, counted over every sequence), warp w
takes [b(w), b(w + 1)), b(w) = min{g : F(g) * W >= w * F(T)}, and tile g
belongs to warp floor(F(g) * W / F(T)); the split applies when no sequence is
left out and F(T) >= 3 W, else the equal split floor(w * T / W).  These tests
pin the properties the kernels rely on: the ranges tile [0, T) in order, none
is empty under the cost split (so a cut unit's contributors are consecutive
warps), the warp-of formula agrees with the ranges, the per-warp cost is even
to within one unit's cost, and a range crossing fewer unit starts gets more
tiles.
"""

from __future__ import annotations

import numpy as np
import pytest

COST = 1  # kStreamUnitCost


def split_start(pre, khg, w, W, FT):
    T = int(pre[-1])
    if FT == 0:
        return (w * T) // W
    target = -(-(w * FT) // W)
    nd = len(pre) - 1
    cu = COST * khg
    if pre[nd] + cu * nd <= target:
        return T
    lo, hi = 0, nd
    while hi - lo > 1:
        mid = (lo + hi) // 2
        if pre[mid] + cu * mid <= target:
            lo = mid
        else:
            hi = mid
    off = target - (pre[lo] + cu * lo)
    ut = (pre[lo + 1] - pre[lo]) // khg
    if ut == 0:
        return int(pre[lo + 1])
    k, t = divmod(off, ut + COST)
    x = (k + 1) * ut if t >= ut else k * ut + t
    return int(min(pre[lo + 1], pre[lo] + x))


def F(pre, khg, g):
    s = int(np.searchsorted(pre, g, "right") - 1)
    while pre[s + 1] == pre[s]:
        s += 1
    ut = (pre[s + 1] - pre[s]) // khg
    return int(g + COST * (khg * s + (g - pre[s]) // ut))


def make(ctx, khg):
    ut = -(-np.asarray(ctx) // 16)
    return np.concatenate([[0], np.cumsum(ut * khg)]).astype(np.int64)


def plan(pre, khg, W, left_out=False):
    nd = len(pre) - 1
    FT = int(pre[-1]) + COST * khg * nd
    return FT if (not left_out and FT >= 3 * W) else 0


@pytest.mark.parametrize("seed", range(24))
def test_ranges_are_nonempty_consecutive_and_balanced(seed):
    rng = np.random.default_rng(seed)
    nd = int(rng.integers(1, 400))
    khg = int(rng.choice([1, 2, 4, 8]))
    ctx = rng.integers(1, 40, nd) if seed % 3 == 0 else rng.integers(1, 3000, nd)
    pre = make(ctx, khg)
    T = int(pre[-1])
    W = int(rng.integers(1, min(3000, max(2, T))))
    FT = plan(pre, khg, W)
    b = [split_start(pre, khg, w, W, FT) for w in range(W + 1)]
    assert b[0] == 0 and b[-1] == T
    assert all(b[w] <= b[w + 1] for w in range(W))
    if FT == 0:
        return
    assert all(b[w] < b[w + 1] for w in range(W)), "an empty range under the cost split"
    for g in rng.integers(0, T, 200):
        w = min(W - 1, F(pre, khg, int(g)) * W // FT)
        assert b[w] <= g < b[w + 1]
    cost = [(F(pre, khg, b[w + 1]) if b[w + 1] < T else FT) - F(pre, khg, b[w]) for w in range(W)]
    assert max(cost) - min(cost) <= 2 * COST + 2


def test_config2_shape_gives_fewer_tiles_to_ranges_that_cross_units():
    """Config 2's shape (256 sequences of U[128, 2048] tokens, 2 KV heads) on
    2368 warps: a range that crosses a unit start holds about one tile less."""
    rng = np.random.default_rng(0)
    ctx = rng.integers(128, 2049, 256)
    pre = make(ctx, 2)
    W = 2368
    FT = plan(pre, 2, W)
    assert FT > 0
    b = [split_start(pre, 2, w, W, FT) for w in range(W + 1)]
    starts = set()
    for s in range(256):
        ut = (pre[s + 1] - pre[s]) // 2
        starts.update({int(pre[s]), int(pre[s] + ut)})
    crossing = [any(b[w] < u < b[w + 1] for u in (x for x in starts if b[w] < x < b[w + 1])) for w in range(W)]
    tiles = np.diff(b)
    cross = np.array(crossing)
    assert tiles[cross].mean() < tiles[~cross].mean() - 0.5


def test_left_out_sequences_use_the_equal_split():
    pre = make([100, 0, 300], 2)
    assert plan(pre, 2, 4, left_out=True) == 0
