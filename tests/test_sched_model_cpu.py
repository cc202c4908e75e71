"""The scheduled decode's work split, checked on the CPU (no GPU needed).

tests/sched_model.py restates the schedule kernel and the decode kernel's
arithmetic structure.  Here, for batches of many shapes (short and long units,
units spanning many CTAs, fewer tiles than CTAs, sequences left out, bad block
ids, several head groups per KV head): every index the kernels form lies in its
buffer, every tile of every good unit is listed exactly once, and the decode's
merge structure (consumer states per piece, partial states of cut units merged
in CTA order) reproduces direct attention.
"""

import numpy as np
import pytest

import sched_model as SM


def _case(seed, ctx, kh, g, d=64, bs=16, ctas=148, nc=8, stages=5, bad_block=None):
    rng = np.random.default_rng(seed)
    ns = len(ctx)
    max_blocks = max(1, max(-(-max(c, 1) // bs) for c in ctx))
    need = sum(-(-max(c, 0) // bs) for c in ctx)
    nb = need + 4
    perm = rng.permutation(nb)
    bt = np.full((ns, max_blocks), -1, dtype=np.int64)
    o = 0
    for s, c in enumerate(ctx):
        k = -(-max(c, 0) // bs)
        bt[s, :k] = perm[o:o + k]
        o += k
    if bad_block is not None:
        bt[bad_block] = nb + 7
    hg = -(-g // 16)
    sch = SM.schedule(ctx, bt, kh, hg, bs, nb, ctas, nc, stages)
    lay = SM.sched_layout(ns, kh, hg, max_blocks, bs, ctas)
    SM.check_bounds(sch, lay["max_tiles"], lay["max_pieces"], ctas, nc, stages)
    # every tile of every good unit once
    seen = {}
    for c, (pbase, np_, r0, n) in enumerate(sch["rec"]):
        for pos in range(np_):
            (s, k, t0, ln), (v0, cx, c0, w) = sch["pieces"][pbase + pos]
            for i in range(ln):
                key = (s, k, t0 + i)
                assert key not in seen
                seen[key] = r0 + v0 + i
    want = {(s, k, t) for s, c in enumerate(ctx) if 1 <= c and -(-c // bs) <= max_blocks
            for k in range(kh * hg) for t in range(-(-c // 16))}
    assert set(seen) == want
    q = rng.standard_normal((ns, kh * g, d)).astype(np.float32)
    kc = rng.standard_normal((nb, kh, bs, d)).astype(np.float32)
    vc = rng.standard_normal((nb, kh, bs, d)).astype(np.float32)
    out = SM.decode(sch, q, kc, vc, kh, hg, bs, 1.0 / np.sqrt(d), nc)
    # direct attention
    for s, c in enumerate(ctx):
        if c < 1 or s == bad_block:
            continue
        toks = [int(bt[s, t // bs]) * bs + t % bs for t in range(c)]
        for h in range(kh * g):
            kvh = h // g
            kk = kc[:, kvh].reshape(-1, d)[toks].astype(np.float64)
            vv = vc[:, kvh].reshape(-1, d)[toks].astype(np.float64)
            x = kk @ q[s, h].astype(np.float64) / np.sqrt(d)
            p = np.exp(x - x.max())
            np.testing.assert_allclose(out[s, h], p @ vv / p.sum(), rtol=1e-9, atol=1e-9)
    return sch




@pytest.mark.parametrize("seed,ns,lo,hi", [(0, 24, 128, 2048), (1, 40, 1, 40), (2, 3, 1, 5), (3, 5, 3000, 9000)])
def test_random_batches(seed, ns, lo, hi):
    rng = np.random.default_rng(100 + seed)
    ctx = rng.integers(lo, hi + 1, ns).tolist()
    _case(seed, ctx, kh=2, g=7, ctas=37)


def test_fewer_tiles_than_ctas():
    sch = _case(5, [1, 17, 5], kh=2, g=7, ctas=148)
    assert sch["ctas"] == sch["T"] == 2 * (1 + 2 + 1)


def test_units_spanning_many_ctas_and_head_groups():
    _case(6, [4000, 33], kh=1, g=20, ctas=16)  # two head groups per KV head


def test_left_out_sequences_and_bad_block_ids():
    sch = _case(7, [50, 0, 300, -3, 700], kh=2, g=4, ctas=9, bad_block=2)
    assert sch["bad"] == [1, 3]
    assert sch["err"] & SM._flag_bits()[2]


def test_head_dim_128_layout():
    _case(8, [1500, 260, 16, 2048], kh=8, g=4, d=128, ctas=11, nc=6, stages=4)


def test_more_pieces_than_the_sort_bound():
    """Past kSchedSortMax pieces per CTA the whole units stay in unit order."""
    rng = np.random.default_rng(9)
    ctx = rng.integers(1, 17, 600).tolist()
    sch = _case(9, ctx, kh=2, g=7, ctas=2)
    assert max(r[1] for r in sch["rec"]) > SM.SORT_MAX
