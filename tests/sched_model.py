"""CPU model of the scheduled decode (variant "sched"): the schedule kernel's
output and the decode kernel's work split, restated in Python.

Test infrastructure only.  ``schedule`` restates decode_schedule_kernel
(csrc/decode_sched.cu): the tile stream of every (sequence, KV head, head
group) unit in sequence order, one contiguous range per CTA
(R(c) = c * T // ctas), each range's pieces in processing order (the piece cut
by the range's end first, the piece cut by its start second, then the whole
units longest first) and the pool row of each tile.  ``decode`` restates the decode kernel's arithmetic structure in float64:
consumer c of a CTA takes the range's tiles c, c + NC, ...; the consumer states
of a piece are merged in consumer order; a cut unit's partial states are merged
in CTA order.  The tests compare the device schedule with ``schedule`` entry by
entry and check ``decode`` against direct attention, which pins the cut-unit
bookkeeping (first CTA, contributor count, partial slots) on the CPU.
"""

from __future__ import annotations

from typing import Dict, List, Optional

import numpy as np

SORT_MAX = 256  # kSchedSortMax


def _flag_bits():
    from mini_vllm_b200 import _native

    return _native.DEV_KV_LEN, _native.DEV_TABLE_SHORT, _native.DEV_BLOCK_ID


def seq_error(ctx: int, block_size: int, max_blocks: int, bits) -> int:
    if ctx < 1:
        return bits[0]
    if -(-ctx // block_size) > max_blocks:
        return bits[1]
    return 0


def schedule(ctx, block_tables, num_kv_heads: int, head_groups: int, block_size: int, num_blocks: int,
             ctas: int, nc: int, stages: int, bits=None) -> Dict:
    """Everything decode_schedule_kernel writes, as Python values.

    Returns {"T", "ctas" (with work), "bad" [seq], "bad_bits", "err",
    "rec": [(pbase, np, r0, n)] per CTA of the grid, "pieces": [(d0, d1)] in
    global order, "rows": {position: row}, "rows0": [[...]] per CTA}."""
    bits = bits or _flag_bits()
    ctx = [int(c) for c in ctx]
    ns = len(ctx)
    ups = num_kv_heads * head_groups
    max_blocks = block_tables.shape[1] if block_tables is not None else 0
    t_seq, good, err = [], [], 0
    for c in ctx:
        e = seq_error(c, block_size, max_blocks, bits[:2])
        err |= e
        good.append(e == 0)
        t_seq.append(0 if e else -(-c // 16))
    pseq = [0]
    for s in range(ns):
        pseq.append(pseq[-1] + t_seq[s] * ups)
    T = pseq[-1]
    gseq = [0]
    for s in range(ns):
        gseq.append(gseq[-1] + (1 if good[s] else 0))
    Ce = min(ctas, T)
    bad = [s for s in range(ns) if not good[s]]
    R = lambda c: c * T // Ce
    cta_of = lambda x: -(-((x + 1) * Ce) // T) - 1

    def locate(x):
        s = max(i for i in range(ns) if pseq[i] <= x)  # the last sequence starting at or before x
        t = t_seq[s]
        k = (x - pseq[s]) // t
        return s, k, t, pseq[s] + k * t

    units = [(s, k) for s in range(ns) if good[s] for k in range(ups)]  # good units in stream order
    rec, pieces, rows, rows0 = [], [], {}, []
    pbase = 0
    for c in range(ctas):
        if c >= Ce:
            rec.append((0, 0, 0, 0))
            rows0.append(None)
            continue
        r0, r1 = R(c), R(c + 1)
        sa, ka, ta, pa = locate(r0)
        sb, kb, tb, pb = locate(r1 - 1)
        gua = gseq[sa] * ups + ka
        np_ = gseq[sb] * ups + kb - gua + 1
        cut_s, cut_e = pa < r0, pb + tb > r1
        info = []
        for i in range(np_):
            s, k = units[gua + i]
            t = t_seq[s]
            P = pseq[s] + k * t
            info.append((s, k, t, P, max(P, r0), min(P + t, r1)))
        # processing order: the piece cut by the range's end, the piece cut by
        # its start, then whole units longest first (ties in unit order; unit
        # order past SORT_MAX pieces)
        if np_ == 1:
            head = [0]
        else:
            head = ([np_ - 1] if cut_e else []) + ([0] if cut_s else [])
        whole = [i for i in range(np_) if i not in head]
        if np_ <= SORT_MAX:
            whole.sort(key=lambda i: (-(info[i][5] - info[i][4]), i))
        order = head + whole
        mine = [None] * np_
        v = 0
        for pos, i in enumerate(order):
            s, k, t, P, ps, pe = info[i]
            c0, w = -1, 0
            if P < r0 or P + t > r1:
                c0 = cta_of(P)
                c1 = cta_of(P + t - 1)
                w = ((c1 - c0 + 1) << 1) | (1 if P == R(c0) else 0)
            mine[pos] = ((s, k, ps - P, pe - ps), (v, ctx[s], c0, w))
            v += pe - ps
        r0s = [-1] * (nc * stages)
        for (d0, d1) in mine:
            s, k, t0, ln = d0
            v0 = d1[0]
            kvh = k // head_groups
            for i in range(ln):
                tok = (t0 + i) * 16
                bi = tok // block_size
                b = int(block_tables[s, bi])
                if 0 <= b < num_blocks:
                    row = (b * num_kv_heads + kvh) * block_size + (tok - bi * block_size)
                else:
                    row = -1
                    err |= bits[2]
                j = v0 + i
                rows[r0 + j] = row
                if j // nc < stages:
                    r0s[(j % nc) * stages + j // nc] = row
        rec.append((pbase, np_, r0, r1 - r0))
        pieces.extend(mine)
        rows0.append(r0s)
        pbase += np_
    return {"T": T, "ctas": Ce, "bad": bad, "bad_bits": err & (bits[0] | bits[1]), "err": err, "rec": rec,
            "pieces": pieces, "rows": rows, "rows0": rows0, "ups": ups}


def check_bounds(sch: Dict, max_tiles: int, max_pieces: int, grid: int, nc: int, stages: int) -> None:
    """Every index the two kernels form from this schedule lies inside its
    buffer (the workspace sizes of sched_layout)."""
    assert len(sch["pieces"]) <= max_pieces
    assert sch["T"] <= max_tiles
    assert nc * stages <= 44
    for c, (pbase, np_, r0, n) in enumerate(sch["rec"]):
        if np_ == 0:
            continue
        assert 0 <= pbase and pbase + np_ <= len(sch["pieces"])
        assert 0 <= r0 and r0 + n <= sch["T"]
        covered = []
        for pos in range(np_):
            d0, d1 = sch["pieces"][pbase + pos]
            assert d0[3] >= 1
            covered.append((d1[0], d1[0] + d0[3]))
            if d1[2] >= 0:
                c0, ncon, first = d1[2], d1[3] >> 1, d1[3] & 1
                assert 0 <= c0 <= c < c0 + ncon <= grid and ncon >= 2
                slot = 2 * c0 + (0 if first else 1) if c == c0 else 2 * c
                assert 0 <= slot < 2 * grid
        # the pieces tile the range in processing order, without gaps or overlaps
        assert covered[0][0] == 0 and covered[-1][1] == n
        assert all(covered[i][1] == covered[i + 1][0] for i in range(len(covered) - 1))


def decode(sch: Dict, q: np.ndarray, kc: np.ndarray, vc: np.ndarray, num_kv_heads: int, head_groups: int,
           block_size: int, scale: float, nc: int) -> np.ndarray:
    """The decode kernel's arithmetic structure in float64: returns out
    [num_seqs, H, D] (rows of left-out sequences zero)."""
    ns, H, D = q.shape
    G = H // num_kv_heads
    out = np.zeros((ns, H, D))
    part: Dict[int, tuple] = {}
    arrivals: Dict[int, int] = {}
    grid = len(sch["rec"])
    for c, (pbase, np_, r0, n) in enumerate(sch["rec"]):
        for pos in range(np_):
            (s, k, t0, ln), (v0, ctx, c0, w) = sch["pieces"][pbase + pos]
            kvh, hg = divmod(k, head_groups)
            h0, nh = kvh * G + hg * 16, min(16, G - hg * 16)
            qs = q[s, h0:h0 + nh].astype(np.float64)
            states = []
            for cc in range(nc):  # consumer cc's tiles of the piece
                js = [j for j in range(v0, v0 + ln) if j % nc == cc]
                if not js:
                    continue
                toks = []
                for j in js:
                    row = sch["rows"][r0 + j]
                    t = t0 + (j - v0)
                    valid = min(16, ctx - t * 16)
                    if row >= 0:
                        toks.extend(row + i for i in range(valid))
                if not toks:
                    continue
                kk = kc.reshape(-1, D)[toks].astype(np.float64)
                vv = vc.reshape(-1, D)[toks].astype(np.float64)
                x = qs @ kk.T * scale
                m = x.max(axis=1)
                p = np.exp(x - m[:, None])
                states.append((m, p.sum(axis=1), p @ vv))
            M, L, O = _merge(states, nh, D)
            if c0 < 0:
                out[s, h0:h0 + nh] = _normalise(L, O)
                continue
            ncon, first = w >> 1, w & 1
            slot_of = lambda cta: 2 * c0 + (0 if first else 1) if cta == c0 else 2 * cta
            part[slot_of(c)] = (M, L, O)
            arrivals[c0] = arrivals.get(c0, 0) + 1
            if arrivals[c0] == ncon:
                _, Lm, Om = _merge([part[slot_of(c0 + i)] for i in range(ncon)], nh, D)
                out[s, h0:h0 + nh] = _normalise(Lm, Om)
    return out


def _merge(states, nh: int, D: int):
    """(M, L, O) of a set of online-softmax states; states without a token
    (M = -inf: every tile's block id was bad) weigh nothing."""
    states = [st for st in states if np.isfinite(st[0]).all()]
    if not states:
        return np.full(nh, -np.inf), np.zeros(nh), np.zeros((nh, D))
    M = np.max([st[0] for st in states], axis=0)
    L = sum(st[1] * np.exp(st[0] - M) for st in states)
    O = sum(st[2] * np.exp(st[0] - M)[:, None] for st in states)
    return M, L, O


def _normalise(L, O):
    return np.where(L[:, None] > 0, O / np.where(L > 0, L, 1.0)[:, None], 0.0)


def sched_layout(num_seqs: int, num_kv_heads: int, head_groups: int, max_blocks: int, block_size: int,
                 ctas: int, G: int = 16, head_dim: int = 64) -> Dict[str, int]:
    """sched_layout (csrc/decode_sched.cu): the bounds on tiles and pieces and
    the workspace offsets of the header, records, pieces, rows, left-out
    list, arrival counters and partial states."""
    units = num_seqs * num_kv_heads * head_groups
    unit_tiles = -(-(max_blocks * block_size) // 16)
    up = lambda v: -(-v // 256) * 256
    mg = min(G, 16)
    lay = {"max_tiles": units * unit_tiles, "max_pieces": units + ctas, "mg": mg, "off_rec": 256}
    lay["off_desc"] = lay["off_rec"] + up(ctas * 256)
    lay["off_rows"] = lay["off_desc"] + up(lay["max_pieces"] * 32)
    lay["off_bad"] = lay["off_rows"] + up(lay["max_tiles"] * 4)
    lay["off_ucnt"] = lay["off_bad"] + up(num_seqs * 4)
    lay["off_part"] = lay["off_ucnt"] + up(ctas * 4)
    lay["bytes"] = lay["off_part"] + up(2 * ctas * mg * (head_dim + 4) * 4)
    return lay
