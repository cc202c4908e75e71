"""Paged gather (prefill prefix read) and prefill attention on the GPU.

The gather is a copy, so it must be bit-exact: against the reference's own
gather_paged_kv outputs (golden vectors), against the oracle's gather for
batched, ragged and shuffled tables, and for every dtype.  Ports the
reference's TestGatherPrefix (test_paged_attention_gpu.py:695-790), its
TestPrefillAttention / TestFutureTokenLeakage (test_paged_attention_ref.py:
342-533), and adds the error contract.

Prefill attention compares with a float32 SDPA of the oracle-gathered K/V
within 2e-3 + 1e-2 * |ref| (bf16 / f16 inputs; the attention itself is torch
SDPA on the GPU in the input dtype).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import make_golden as MG
import mini_vllm_b200 as M
import oracle
from conftest import np_to_torch, torch_to_np

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
TDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def _pool(nb, kh, bs, d, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    kc = torch.randn(nb, kh, bs, d, generator=g).to(dtype).to(DEV)
    vc = torch.randn(nb, kh, bs, d, generator=g).to(dtype).to(DEV)
    return kc, vc


def _oracle_gather(kc, vc, ids, n, bs, dt):
    return oracle.gather(torch_to_np(kc, dt), torch_to_np(vc, dt), np.asarray(ids, np.int64), n, bs, dt)


def test_golden_gathers_bit_exact(golden):
    """Every gather case of the reference's own gather_paged_kv, bit for bit."""
    cases, arrays = golden
    ran = 0
    for c in [c for c in cases if c["kind"] == "gather"]:
        x = MG.gather_inputs(c)
        kc, vc = np_to_torch(x["kc"], c["dtype"], DEV), np_to_torch(x["vc"], c["dtype"], DEV)
        if c["expect_error"]:
            with pytest.raises(IndexError, match="insufficient"):
                M.gather_paged_kv(kc, vc, x["table"].tolist(), c["num_tokens"], c["block_size"])
            continue
        k, v = M.gather_paged_kv(kc, vc, x["table"].tolist(), c["num_tokens"], c["block_size"])
        assert k.shape == (c["num_tokens"], c["num_kv_heads"], c["head_dim"]) and k.dtype == TDT[c["dtype"]]
        assert np.array_equal(torch_to_np(k, c["dtype"]), arrays[f"{c['name']}/k"])
        assert np.array_equal(torch_to_np(v, c["dtype"]), arrays[f"{c['name']}/v"])
        ran += 1
    assert ran >= 6


# ---- TestGatherPrefix (test_paged_attention_gpu.py:695-790) ----
def _written_pool(nb, seq_len, slots, seed):
    kc = torch.zeros(nb, 2, 16, 64, dtype=torch.float16, device=DEV)
    vc = torch.zeros_like(kc)
    g = torch.Generator().manual_seed(seed)
    k = (torch.randn(seq_len, 2, 64, generator=g) + 10.0).to(torch.float16).to(DEV)
    v = (torch.randn(seq_len, 2, 64, generator=g) + 1000.0).to(torch.float16).to(DEV)
    M.paged_cache_write(k, v, kc, vc, torch.as_tensor(slots, dtype=torch.int64, device=DEV), 16)
    return kc, vc, k, v


@pytest.mark.parametrize("seq_len,nb,table", [(10, 32, [0]), (25, 32, [0, 1])])
def test_gather_prefix_full_and_multi_block(seq_len, nb, table):
    kc, vc, k, v = _written_pool(nb, seq_len, list(range(seq_len)), seed=seq_len)
    bt = torch.tensor([table], dtype=torch.int64, device=DEV)
    gk, gv = M.gather_prefix_kv(kc, vc, bt, [seq_len], [0], 16)
    assert torch.equal(gk, k) and torch.equal(gv, v)
    rk, rv = _oracle_gather(kc, vc, table, seq_len, 16, "f16")
    assert np.array_equal(torch_to_np(gk, "f16"), rk) and np.array_equal(torch_to_np(gv, "f16"), rv)


def test_gather_prefix_noncontiguous_blocks():
    slots = list(range(160, 176)) + list(range(800, 804))
    kc, vc, k, v = _written_pool(64, 20, slots, seed=3)
    bt = torch.tensor([[10, 50]], dtype=torch.int64, device=DEV)
    gk, gv = M.gather_prefix_kv(kc, vc, bt, [20], [0], 16)
    assert torch.equal(gk, k) and torch.equal(gv, v)


def test_gather_prefix_zero_returns_empty():
    kc, vc = _pool(32, 2, 16, 64, torch.float16, 1)
    gk, gv = M.gather_prefix_kv(kc, vc, torch.zeros(1, 1, dtype=torch.int64, device=DEV), [0], [0], 16)
    assert gk.shape == (0, 2, 64) and gv.shape == (0, 2, 64)


# ---- batched, ragged, every dtype ----
@pytest.mark.parametrize("dt,bs,d,kh", [("bf16", 16, 64, 2), ("f16", 32, 128, 8), ("f32", 1, 64, 1),
                                        ("bf16", 8, 128, 4), ("f32", 16, 64, 2), ("f32", 64, 128, 1),
                                        ("bf16", 64, 256, 3), ("f16", 16, 8, 2), ("bf16", 16, 64, 6)])
def test_batched_gather_matches_oracle(dt, bs, d, kh):
    rng = np.random.default_rng(bs * 1000 + d)
    nseq_table = 12
    counts = rng.integers(0, 300, size=nseq_table)
    counts[3] = 0
    need = [(int(n) + bs - 1) // bs for n in counts]
    maxb = max(need) + 2
    nb = sum(need) + 5
    perm = rng.permutation(nb)
    table = np.full((nseq_table, maxb), -1, np.int64)
    pos = 0
    for i, k in enumerate(need):
        table[i, :k] = perm[pos:pos + k]
        pos += k
    kc, vc = _pool(nb, kh, bs, d, TDT[dt], seed=bs + d)
    seqs = [7, 0, 3, 11, 5, 5]  # repeats and a zero-length sequence are allowed
    gk, gv = M.gather_prefix_kv(kc, vc, torch.from_numpy(table).to(DEV), [int(counts[s]) for s in seqs], seqs, bs)
    off = 0
    for s in seqs:
        n = int(counts[s])
        rk, rv = _oracle_gather(kc, vc, table[s, :need[s]], n, bs, dt)
        assert np.array_equal(torch_to_np(gk[off:off + n], dt), rk), f"seq {s}"
        assert np.array_equal(torch_to_np(gv[off:off + n], dt), rv), f"seq {s}"
        off += n
    assert off == gk.shape[0]


def test_large_batched_gather_checksum():
    """64 sequences of up to 4096 tokens (one launch, ~70 MB moved), against a
    torch index-gather of the same rows."""
    rng = np.random.default_rng(5)
    counts = rng.integers(1, 4096, size=64)
    need = (counts + 15) // 16
    nb = int(need.sum()) + 8
    perm = rng.permutation(nb)
    maxb = int(need.max())
    table = np.full((64, maxb), -1, np.int64)
    pos = 0
    for i, k in enumerate(need):
        table[i, :k] = perm[pos:pos + k]
        pos += k
    kc, vc = _pool(nb, 2, 16, 64, torch.bfloat16, seed=9)
    bt = torch.from_numpy(table).to(DEV)
    gk, gv = M.paged_gather(kc, vc, bt, list(range(64)), counts.tolist(), 16)
    rows, toks = [], []
    for i, n in enumerate(counts.tolist()):
        p = torch.arange(n, device=DEV)
        rows.append(bt[i][p // 16])
        toks.append(p % 16)
    blk, tok = torch.cat(rows), torch.cat(toks)
    assert torch.equal(gk, kc[blk, :, tok, :]) and torch.equal(gv, vc[blk, :, tok, :])


# ---- the C ABI: zero rows and error bits ----
def _abi_gather(kc, vc, bt, rows, offsets, total, counter=None):
    """mvb_paged_gather with explicit (possibly inconsistent) offsets and an
    optional work counter; returns (status, K, V, error word).  The outputs
    start filled with 7.0."""
    from mini_vllm_b200 import _native

    nb, kh, bs, d = kc.shape
    meta = torch.tensor(list(rows) + list(offsets), dtype=torch.int64, device=DEV)
    ko = torch.full((total, kh, d), 7.0, dtype=kc.dtype, device=DEV)
    vo = torch.full_like(ko, 7.0)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    st = _native.lib().mvb_paged_gather(
        kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), bt.shape[0], bt.stride(0), bt.shape[1], meta.data_ptr(),
        meta.data_ptr() + 8 * len(rows), ko.data_ptr(), vo.data_ptr(), len(rows), total, kh, d, bs, nb,
        {torch.bfloat16: _native.DTYPE_BF16, torch.float16: _native.DTYPE_F16,
         torch.float32: _native.DTYPE_F32}[kc.dtype], None if counter is None else counter.data_ptr(),
        err.data_ptr(), torch.cuda.current_stream(DEV).cuda_stream)
    torch.cuda.synchronize()
    return st, ko, vo, int(err.item())


def _expected(kc, vc, bt, rows, offsets, total):
    """Token t of sequence i (offsets[i] <= t < offsets[i + 1]) is
    cache[bt[rows[i]][p // BS], :, p % BS]; a token without a sequence, or
    whose block is -1 / past the pool / past the table, is a zero row."""
    nb, kh, bs, d = kc.shape
    ek = torch.zeros(total, kh, d, dtype=kc.dtype, device=DEV)
    ev = torch.zeros_like(ek)
    for i, r in enumerate(rows):
        for t in range(max(offsets[i], 0), min(offsets[i + 1], total)):
            p = t - offsets[i]
            if not 0 <= r < bt.shape[0] or p // bs >= bt.shape[1]:
                continue
            b = int(bt[r, p // bs])
            if 0 <= b < nb:
                ek[t], ev[t] = kc[b, :, p % bs], vc[b, :, p % bs]
    return ek, ev


@pytest.mark.parametrize("with_counter", [False, True])
@pytest.mark.parametrize("dt,bs,d,kh", [("bf16", 16, 64, 2), ("f32", 8, 64, 2)])  # tile form, vector form
def test_abi_bad_blocks_give_zero_rows(dt, bs, d, kh, with_counter):
    kc, vc = _pool(12, kh, bs, d, TDT[dt], 4)
    bt = torch.tensor([[3, -1, 5, 1], [2, 99, 7, 0], [4, 6, 8, 9]], dtype=torch.int64, device=DEV)
    rows, counts = [0, 1, 2, 5], [3 * bs + 5, 2 * bs + 1, 4 * bs, 7]  # row 5 is outside the table
    offsets = [0]
    for n in counts:
        offsets.append(offsets[-1] + n)
    counter = torch.zeros(2, dtype=torch.int32, device=DEV) if with_counter else None
    st, ko, vo, err = _abi_gather(kc, vc, bt, rows, offsets, offsets[-1], counter)
    assert st == 0
    ek, ev = _expected(kc, vc, bt, rows, offsets, offsets[-1])
    assert torch.equal(ko, ek) and torch.equal(vo, ev)
    assert err & 2  # MVB_DEV_BLOCK_ID
    if with_counter:
        assert counter.tolist() == [0, 0]


@pytest.mark.parametrize("short_by", [0, 3])
def test_abi_batch_above_the_staged_sequence_limit(short_by):
    """1100 short sequences (0-8 tokens): the offset check takes several
    rounds per warp and the sequence search three ballot levels.
    short_by > 0: offsets end before total_tokens, and the tail rows are zero
    with MVB_DEV_KV_LEN."""
    rng = np.random.default_rng(33)
    counts = [int(c) for c in rng.integers(0, 9, size=1100)]
    need = [max(1, (c + 15) // 16) for c in counts]
    nb = sum(need) + 2
    perm = torch.from_numpy(rng.permutation(nb)).to(DEV)
    bt = torch.zeros((1100, 1), dtype=torch.int64, device=DEV)
    bt[:, 0] = perm[:1100]
    kc, vc = _pool(nb, 2, 16, 64, torch.bfloat16, 9)
    offsets = [0]
    for n in counts:
        offsets.append(offsets[-1] + n)
    total = offsets[-1] + short_by
    counter = torch.zeros(2, dtype=torch.int32, device=DEV)
    st, ko, vo, err = _abi_gather(kc, vc, bt, list(range(1100)), offsets, total, counter)
    assert st == 0 and counter.tolist() == [0, 0]
    rows = torch.cat([torch.full((n,), i, dtype=torch.int64) for i, n in enumerate(counts)]).to(DEV)
    tok = torch.cat([torch.arange(n) for n in counts]).to(DEV)
    blk = bt[rows, 0]
    ek = torch.zeros((total, 2, 64), dtype=torch.bfloat16, device=DEV)
    ev = torch.zeros_like(ek)
    ek[:offsets[-1]], ev[:offsets[-1]] = kc[blk, :, tok, :], vc[blk, :, tok, :]
    assert torch.equal(ko, ek) and torch.equal(vo, ev)
    assert (err & 1) == (1 if short_by else 0)


def test_abi_work_counter_is_left_zero_and_results_repeat():
    """With the work counter the tail of the copy is handed out at run time,
    so warps take different items from call to call; the output must not
    change, and the two words must be zero after every call."""
    rng = np.random.default_rng(21)
    counts = [int(c) for c in rng.integers(1, 1500, size=96)]
    need = [(c + 15) // 16 for c in counts]
    nb = sum(need) + 3
    perm = torch.from_numpy(rng.permutation(nb)).to(DEV)
    bt = torch.full((96, max(need)), -1, dtype=torch.int64, device=DEV)
    pos = 0
    for i, k in enumerate(need):
        bt[i, :k] = perm[pos:pos + k]
        pos += k
    kc, vc = _pool(nb, 2, 16, 64, torch.bfloat16, 8)
    offsets = [0]
    for n in counts:
        offsets.append(offsets[-1] + n)
    counter = torch.zeros(2, dtype=torch.int32, device=DEV)
    st, k0, v0, err = _abi_gather(kc, vc, bt, list(range(96)), offsets, offsets[-1])  # static split
    assert st == 0 and err == 0
    for _ in range(3):
        st, k1, v1, err = _abi_gather(kc, vc, bt, list(range(96)), offsets, offsets[-1], counter)
        assert st == 0 and err == 0
        assert torch.equal(k1, k0) and torch.equal(v1, v0)
        assert counter.tolist() == [0, 0]


@pytest.mark.parametrize("offsets,total", [([0, 20, 50], 64), ([5, 30, 50], 50), ([0, 40, 30, 70], 70)])
def test_abi_offsets_that_are_not_a_prefix_sum(offsets, total):
    """Offsets that end short of total_tokens, start past 0, or fall: the tile
    form hands over to the per-token loop.  With rising offsets a token
    without a sequence is a zero row with MVB_DEV_KV_LEN; with falling ones
    the token-to-sequence search is not defined, but every row is written."""
    kc, vc = _pool(24, 2, 16, 64, torch.bfloat16, 5)
    bt = torch.arange(24, dtype=torch.int64, device=DEV).flip(0).reshape(3, 8).contiguous()
    rows = list(range(len(offsets) - 1))
    st, ko, vo, err = _abi_gather(kc, vc, bt, rows, offsets, total)
    assert st == 0
    if all(a <= b for a, b in zip(offsets, offsets[1:])):
        ek, ev = _expected(kc, vc, bt, rows, offsets, total)
        assert torch.equal(ko, ek) and torch.equal(vo, ev)
        assert err & 1  # MVB_DEV_KV_LEN
    else:
        assert not (ko == 7.0).all(dim=-1).any() and not (vo == 7.0).all(dim=-1).any()


def test_gathers_on_two_streams_at_once():
    """paged_gather keeps one work counter per stream: gathers queued on two
    streams without a sync in between run concurrently and each still returns
    exactly its rows."""
    rng = np.random.default_rng(41)
    cases = []
    for seed in (1, 2):
        counts = [int(c) for c in rng.integers(1, 1200, size=128)]
        need = [(c + 15) // 16 for c in counts]
        nb = sum(need) + 2
        perm = torch.from_numpy(rng.permutation(nb)).to(DEV)
        bt = torch.full((128, max(need)), -1, dtype=torch.int64, device=DEV)
        pos = 0
        for i, k in enumerate(need):
            bt[i, :k] = perm[pos:pos + k]
            pos += k
        kc, vc = _pool(nb, 2, 16, 64, torch.bfloat16, seed)
        rows = torch.cat([torch.full((n,), i, dtype=torch.int64) for i, n in enumerate(counts)]).to(DEV)
        tok = torch.cat([torch.arange(n) for n in counts]).to(DEV)
        blk = bt[rows, tok // 16]
        cases.append((kc, vc, bt, counts, kc[blk, :, tok % 16, :], vc[blk, :, tok % 16, :]))
    streams = [torch.cuda.Stream(DEV), torch.cuda.Stream(DEV)]
    torch.cuda.synchronize()
    outs = [[], []]
    for _ in range(4):
        for i, st in enumerate(streams):
            kc, vc, bt, counts = cases[i][:4]
            with torch.cuda.stream(st):
                outs[i].append(M.paged_gather(kc, vc, bt, list(range(128)), counts, 16, strict=False))
    torch.cuda.synchronize()
    M.check_device_errors(DEV)
    for i in range(2):
        ek, ev = cases[i][4], cases[i][5]
        for gk, gv in outs[i]:
            assert torch.equal(gk, ek) and torch.equal(gv, ev)


# ---- errors ----
def test_gather_errors():
    kc, vc = _pool(8, 2, 16, 64, torch.bfloat16, 2)
    bt = torch.tensor([[0, -1], [1, 2]], dtype=torch.int64, device=DEV)
    with pytest.raises(IndexError, match="out of range"):  # -1 inside the prefix
        M.gather_prefix_kv(kc, vc, bt, [20], [0], 16)
    with pytest.raises(IndexError, match="insufficient"):  # table too short
        M.gather_prefix_kv(kc, vc, bt, [40], [1], 16)
    with pytest.raises(IndexError, match="sequence index"):
        M.gather_prefix_kv(kc, vc, bt, [4], [2], 16)
    bad = torch.tensor([[0, 99]], dtype=torch.int64, device=DEV)  # block id past the pool
    with pytest.raises(IndexError, match="out of range"):
        M.gather_prefix_kv(kc, vc, bad, [30], [0], 16)
    with pytest.raises(ValueError):
        M.gather_prefix_kv(kc, vc, bt, [-1], [0], 16)
    # the error word is left clear after a raised error
    gk, _ = M.gather_prefix_kv(kc, vc, bt, [16], [0], 16)
    assert torch.equal(gk, kc[0].permute(1, 0, 2))


# ---- prefill attention ----
def _sdpa_ref(q, k, v, cached, reps):
    """float32 SDPA with the offset causal mask (the reference's math)."""
    qf, kf, vf = q.float(), k.float().repeat_interleave(reps, 1), v.float().repeat_interleave(reps, 1)
    kv_len, q_len = kf.shape[0], qf.shape[0]
    mask = torch.arange(kv_len, device=q.device)[None, :] <= torch.arange(cached, cached + q_len,
                                                                          device=q.device)[:, None]
    o = torch.nn.functional.scaled_dot_product_attention(
        qf.permute(1, 0, 2)[None], kf.permute(1, 0, 2)[None], vf.permute(1, 0, 2)[None], attn_mask=mask,
        scale=q.shape[-1] ** -0.5)
    return o[0].permute(1, 0, 2)


def _close(a, b):
    assert ((a.float() - b).abs() <= 2e-3 + 1e-2 * b.abs()).all()


def _prefill_setup(dtype, seqs, bs=16, kh=2, h=14, d=64, seed=0):
    """Write each sequence's whole context (cached + new) into a shuffled pool."""
    g = torch.Generator().manual_seed(seed)
    need = [(c + n + bs - 1) // bs for c, n in seqs]
    nb = sum(need) + 4
    perm = torch.randperm(nb, generator=g)
    maxb = max(need)
    table = torch.full((len(seqs), maxb), -1, dtype=torch.int64)
    pos = 0
    for i, k in enumerate(need):
        table[i, :k] = perm[pos:pos + k]
        pos += k
    kc = torch.randn(nb, kh, bs, d, generator=g).to(dtype).to(DEV)
    vc = torch.randn(nb, kh, bs, d, generator=g).to(dtype).to(DEV)
    ks, vs, qs, new_k, new_v = [], [], [], [], []
    for i, (c, n) in enumerate(seqs):
        k = torch.randn(c + n, kh, d, generator=g).to(dtype).to(DEV)
        v = torch.randn(c + n, kh, d, generator=g).to(dtype).to(DEV)
        p = torch.arange(c + n)
        slots = (table[i][p // bs] * bs + p % bs).to(DEV)
        M.paged_cache_write(k, v, kc, vc, slots, bs)
        ks.append(k)
        vs.append(v)
        new_k.append(k[c:])
        new_v.append(v[c:])
        qs.append(torch.randn(n, h, d, generator=g).to(dtype).to(DEV))
    backend = M.AttentionBackendB200(M.ModelConfig(num_heads=h, num_kv_heads=kh, head_dim=d))
    pool = M.KVCachePool([kc], [vc], nb, bs, 1, kh, d, DEV, dtype)
    backend._pool = pool
    group = M.AttentionGroup(seq_indices=list(range(len(seqs))), attention_type="prefill_gpu",
                             cached_len_before=torch.tensor([c for c, _ in seqs]),
                             query_len=torch.tensor([n for _, n in seqs]),
                             kv_len_after=torch.tensor([c + n for c, n in seqs]))
    meta = M.AttentionMetadata(groups=[group], prefill_block_tables=table.to(DEV), block_size=bs,
                               num_kv_heads=kh, head_dim=d)
    return backend, pool, meta, ks, vs, qs, torch.cat(new_k), torch.cat(new_v)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("with_chunk", [True, False])
def test_prefill_attention_matches_sdpa(dtype, with_chunk):
    """Full prefill, prefix 8 + 1..3 new tokens, several sequences (the
    reference's TestPrefillAttention cases) and a long chunked prefill."""
    seqs = [(0, 12), (8, 2), (8, 3), (8, 1), (37, 5), (300, 64)]
    backend, pool, meta, ks, vs, qs, nk, nv = _prefill_setup(dtype, seqs)
    q = torch.cat(qs)
    out = backend.prefill_attention(0, q, nk if with_chunk else None, nv if with_chunk else None, meta, pool)
    assert out.shape == q.shape and out.dtype == dtype
    off = 0
    for i, (c, n) in enumerate(seqs):
        _close(out[off:off + n], _sdpa_ref(qs[i], ks[i], vs[i], c, 7))
        off += n


def test_prefill_future_tokens_blocked():
    """TestFutureTokenLeakage (test_paged_attention_ref.py:485-533): a query at
    position P+i never sees positions > P+i, even when they hold extreme V."""
    kc = torch.zeros(4, 1, 4, 8, dtype=torch.float16, device=DEV)  # head_dim 8: 16-byte rows
    vc = torch.zeros_like(kc)
    k_all = torch.zeros(7, 1, 8, dtype=torch.float16)
    v_all = torch.zeros(7, 1, 8, dtype=torch.float16)
    for pos in range(7):
        k_all[pos] = pos + 1
        v_all[pos] = pos + 1
    v_all[5:] = 1e4
    M.paged_cache_write(k_all.to(DEV), v_all.to(DEV), kc, vc, torch.arange(7, device=DEV), 4)
    q = torch.randn(3, 2, 8, generator=torch.Generator().manual_seed(0)).to(torch.float16).to(DEV)
    backend = M.AttentionBackendB200.__new__(M.AttentionBackendB200)  # head_dim 8 is below the decode set
    backend.strict = True
    pool = M.KVCachePool([kc], [vc], 4, 4, 1, 1, 8, DEV, torch.float16)
    group = M.AttentionGroup(seq_indices=[0], attention_type="prefill_gpu", cached_len_before=torch.tensor([4]),
                             query_len=torch.tensor([3]), kv_len_after=torch.tensor([7]))
    meta = M.AttentionMetadata(groups=[group], prefill_block_tables=torch.tensor([[0, 1]], device=DEV),
                               block_size=4, num_kv_heads=1, head_dim=8)
    out = M.AttentionBackendB200.prefill_attention(backend, 0, q, None, None, meta, pool)
    ref = _sdpa_ref(q, k_all.to(DEV), v_all.to(DEV), 4, 2)
    _close(out, ref)
    assert out[0].float().abs().max() < 100  # q0 (position 4) does not see the 1e4 values at 5, 6
