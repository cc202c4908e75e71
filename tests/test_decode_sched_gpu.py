"""The scheduled persistent decode (variant "sched") and its per-step
schedule (GPU).

The schedule kernel cuts the tile stream of every (sequence, KV head, head
group) unit into one range per SM, lists each range's pieces (the ones cut by
its ends first) and resolves the pool row of every tile; the decode kernel
streams each range with self-issuing consumer warps, and the last piece of a
unit cut by a range boundary merges it.  These tests check the device schedule
entry by entry against its CPU restatement (tests/sched_model.py), the decode
against the oracle over batch sizes from 1 to 5000 and units spanning many
SMs, the reuse of one schedule by several layers, the write-then-decode
overlap, the backend's once-per-step build, concurrent streams, and bad
sequences.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import mini_vllm_b200 as M
import oracle
import sched_model as SM
from conftest import torch_to_np
from mini_vllm_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = "cuda"
NC = {64: 11, 128: 6}     # consumer warps per CTA
STAGES = {64: 4, 128: 4}  # ring stages per consumer


def close(gpu: torch.Tensor, ref: np.ndarray, msg: str = ""):
    g = gpu.float().cpu().numpy()
    assert np.isfinite(g).all(), msg
    err = np.abs(g - ref)
    assert (err <= 2e-3 + 1e-2 * np.abs(ref)).all(), f"{msg}: max abs err {err.max():.3e}"


def ref_decode(spec, t, kc=None, vc=None):
    kc = t["key_caches"][0] if kc is None else kc
    vc = t["value_caches"][0] if vc is None else vc
    ref, st = oracle.decode(torch_to_np(t["query"], "bf16"), torch_to_np(kc, "bf16"), torch_to_np(vc, "bf16"),
                            spec.block_tables, spec.context_lens, spec.block_size, "bf16")
    assert (st == 0).all()
    return ref


def _ctas():
    return torch.cuda.get_device_properties(0).multi_processor_count


def read_schedule(sched, spec, h, kh, d):
    """The device schedule: header, records, pieces, rows, left-out list and
    arrival counters, cut out of the workspace at sched_layout's offsets."""
    hg = -(-(h // kh) // 16)
    lay = SM.sched_layout(spec.num_seqs, kh, hg, spec.max_blocks, 16, _ctas(), G=h // kh, head_dim=d)
    ws = sched.workspace.cpu()
    i32 = lambda a, b: ws[a:b].view(torch.int32).numpy()
    hdr = i32(0, 256)
    T, ce, n_bad = int(hdr[0]), int(hdr[1]), int(hdr[2])
    rec = i32(lay["off_rec"], lay["off_rec"] + 256 * _ctas()).reshape(_ctas(), 64)
    npieces = int(rec[:, 1].sum())
    desc = i32(lay["off_desc"], lay["off_desc"] + 32 * npieces).reshape(npieces, 8)
    rows = i32(lay["off_rows"], lay["off_rows"] + 4 * T)
    bad = i32(lay["off_bad"], lay["off_bad"] + 4 * n_bad)
    ucnt = i32(lay["off_ucnt"], lay["off_ucnt"] + 4 * _ctas())
    return {"hdr": hdr, "T": T, "ctas": ce, "rec": rec, "desc": desc, "rows": rows, "bad": bad, "ucnt": ucnt}


def check_schedule(dev, spec, h, kh, d):
    """The device schedule equals the CPU restatement entry by entry."""
    hg = -(-(h // kh) // 16)
    want = SM.schedule(spec.context_lens, spec.block_tables, kh, hg, 16, spec.num_blocks, _ctas(), NC[d], STAGES[d])
    assert dev["T"] == want["T"] and dev["ctas"] == want["ctas"]
    assert dev["bad"].tolist() == want["bad"]
    assert (dev["ucnt"] == 0).all()  # arrival counters at rest
    for c in range(_ctas()):
        assert tuple(dev["rec"][c, :4]) == want["rec"][c], c
        pbase, np_ = want["rec"][c][:2]
        for pos in range(min(np_, 2)):  # the record's copy of its first two pieces
            assert tuple(dev["rec"][c, 4 + 8 * pos:12 + 8 * pos]) == want["pieces"][pbase + pos][0] + \
                want["pieces"][pbase + pos][1]
        if np_:
            assert dev["rec"][c, 20:20 + NC[d] * STAGES[d]].tolist() == want["rows0"][c], c
    got_pieces = [tuple(map(int, r[:4])) + tuple(map(int, r[4:])) for r in dev["desc"]]
    assert got_pieces == [a + b for a, b in want["pieces"]]
    assert dev["rows"].tolist() == [want["rows"][i] for i in range(want["T"])]
    SM.check_bounds(want, SM.sched_layout(spec.num_seqs, kh, hg, spec.max_blocks, 16, _ctas())["max_tiles"],
                    SM.sched_layout(spec.num_seqs, kh, hg, spec.max_blocks, 16, _ctas())["max_pieces"], _ctas(),
                    NC[d], STAGES[d])
    return want


@pytest.mark.parametrize("num_seqs,heads", [(256, (14, 2)), (7, (14, 2)), (96, (32, 8)), (3, (40, 2))])
def test_schedule_matches_the_cpu_restatement(num_seqs, heads):
    h, kh = heads
    d = 128 if kh == 8 else 64
    ctx = W.context_lengths(2, seed=num_seqs, num_seqs=num_seqs)
    if num_seqs == 3:
        ctx[:] = [1, 20000, 33]
    spec = W.build_spec("s", ctx, h, kh, d, 16, seed=1)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    sched = M.build_decode_schedule(t["kv_len"], t["block_tables"], h, kh, d, 16, spec.num_blocks, torch.bfloat16,
                                    variant="sched")
    torch.cuda.synchronize()
    check_schedule(read_schedule(sched, spec, h, kh, d), spec, h, kh, d)


def test_one_schedule_serves_every_layer():
    spec = W.make_spec(2, seed=40)
    t = W.torch_tensors(spec, torch.bfloat16, DEV, num_layers=3)
    sched = M.build_decode_schedule(t["kv_len"], t["block_tables"], 14, 2, 64, 16, spec.num_blocks, torch.bfloat16,
                                    variant="sched")
    for layer in range(3):
        out = M.paged_decode_attention(t["query"], t["key_caches"][layer], t["value_caches"][layer],
                                       t["block_tables"], t["kv_len"], 16, schedule=sched)
        close(out, ref_decode(spec, t, t["key_caches"][layer], t["value_caches"][layer]), f"layer {layer}")
        assert (read_schedule(sched, spec, 14, 2, 64)["ucnt"] == 0).all()  # the last arrivals reset them


@pytest.mark.parametrize("num_seqs", [1, 2, 3, 8, 37, 148, 300, 1500, 5000])
def test_batch_sizes(num_seqs):
    """From one sequence (its units cut across the whole GPU) to thousands
    (many pieces per CTA), twice in a row (the counters the first call left at
    zero)."""
    ctx = W.context_lengths(2, seed=num_seqs, num_seqs=num_seqs)
    if num_seqs <= 3:
        ctx[:] = [3000, 1, 77][:num_seqs]
    spec = W.build_spec("b", ctx, 14, 2, 64, 16, seed=num_seqs)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    ref = ref_decode(spec, t)
    outs = []
    for _ in range(2):
        out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                       t["kv_len"], 16, variant="sched")
        close(out, ref, f"n={num_seqs}")
        outs.append(out)
    assert torch.equal(outs[0], outs[1])  # fixed work split: the same bits every time


@pytest.mark.parametrize("head_dim,heads,kv_heads", [(64, 14, 2), (128, 32, 8)])
def test_long_units_many_ctas(head_dim, heads, kv_heads):
    """Units thousands of tiles long: each spans many CTAs, and the last of
    its pieces to arrive merges them (in rounds of 4 partial states)."""
    ctx = np.array([40000, 5, 30001, 17], np.int64)
    spec = W.build_spec("long", ctx, heads, kv_heads, head_dim, 16, seed=41)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    sched = M.build_decode_schedule(t["kv_len"], t["block_tables"], heads, kv_heads, head_dim, 16, spec.num_blocks,
                                    torch.bfloat16, variant="sched")
    dev = read_schedule(sched, spec, heads, kv_heads, head_dim)
    want = check_schedule(dev, spec, heads, kv_heads, head_dim)
    assert max(d1[3] >> 1 for _, d1 in want["pieces"]) > 4
    ref = ref_decode(spec, t)
    for _ in range(2):
        out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                       t["kv_len"], 16, schedule=sched)
        close(out, ref, f"long D={head_dim}")


def _write_then_decode_case(seed: int, num_seqs: int):
    spec = W.make_spec(2, seed=seed, num_seqs=num_seqs)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    t["new_key"].fill_(4.0)
    t["new_value"].fill_(3.0)
    kc, vc = torch_to_np(t["key_caches"][0], "bf16"), torch_to_np(t["value_caches"][0], "bf16")
    oracle.cache_write(torch_to_np(t["new_key"], "bf16"), torch_to_np(t["new_value"], "bf16"), kc, vc,
                       spec.slot_mapping, 16, "bf16")
    ref, st = oracle.decode(torch_to_np(t["query"], "bf16"), kc, vc, spec.block_tables, spec.context_lens, 16,
                            "bf16")
    assert (st == 0).all()
    return spec, t, ref


@pytest.mark.parametrize("num_seqs", [256, 5])
def test_write_then_decode_with_a_schedule(num_seqs):
    """The bench's step order: schedule, then per layer the KV write and the
    decode with the schedule ready and its inputs read while the write runs.
    The new tokens dominate attention (K = 4, V = 3), so a decode that read
    the cache before the write landed would be far off."""
    spec, t, ref = _write_then_decode_case(33, num_seqs)
    sched = M.build_decode_schedule(t["kv_len"], t["block_tables"], 14, 2, 64, 16, spec.num_blocks, torch.bfloat16,
                                    variant="sched")
    outs = []
    for _ in range(3):
        kc, vc = t["key_caches"][0].clone(), t["value_caches"][0].clone()
        M.paged_cache_write(t["new_key"], t["new_value"], kc, vc, t["slot_mapping"], 16, strict=False,
                            check_duplicates=False)
        o = M.paged_decode_attention(t["query"], kc, vc, t["block_tables"], t["kv_len"], 16, strict=False,
                                     after_write=True, schedule=sched)
        M.check_device_errors()
        close(o, ref, "after_write + schedule")
        outs.append(o)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    # the inline form (schedule built inside the call, after the write) agrees bit for bit
    kc, vc = t["key_caches"][0].clone(), t["value_caches"][0].clone()
    M.paged_cache_write(t["new_key"], t["new_value"], kc, vc, t["slot_mapping"], 16)
    o = M.paged_decode_attention(t["query"], kc, vc, t["block_tables"], t["kv_len"], 16, after_write=True,
                                 variant="sched")
    assert torch.equal(o, outs[0])


def test_backend_builds_the_schedule_once_per_step():
    spec, t, ref = _write_then_decode_case(34, 64)
    backend = M.AttentionBackendB200(M.ModelConfig(num_heads=14, num_kv_heads=2, head_dim=64), strict=True,
                                     overlap_after_write=True, decode_variant="sched")
    L = 3
    kcs = [t["key_caches"][0].clone() for _ in range(L)]
    vcs = [t["value_caches"][0].clone() for _ in range(L)]
    pool = M.KVCachePool(kcs, vcs, spec.num_blocks, 16, L, 2, 64, torch.device(DEV), torch.bfloat16)
    backend._pool = pool

    def meta():
        g = M.AttentionGroup(seq_indices=list(range(spec.num_seqs)), attention_type="decode_gpu",
                             cached_len_before=None, query_len=None, kv_len_after=t["kv_len"])
        return M.AttentionMetadata(groups=[g], decode_block_tables=t["block_tables"], block_size=16,
                                   num_kv_heads=2, head_dim=64)

    first = None
    for step in range(2):
        m = meta()
        for layer in range(L):
            backend.write_kv_cache(layer, t["new_key"], t["new_value"], t["slot_mapping"])
            o = backend.decode_attention(layer, t["query"], m, pool)
            close(o, ref, f"step {step} layer {layer}")
            assert backend._schedule_built_now == (layer == 0)
            if first is None:
                first = o
            assert torch.equal(o, first)


def test_two_streams_at_once():
    """Calls on two streams may overlap: each stream has its own schedule
    workspace (the inline form), so neither disturbs the other's counters."""
    specs = [W.make_spec(2, seed=50 + i, num_seqs=n) for i, n in enumerate((200, 90))]
    ts = [W.torch_tensors(s, torch.bfloat16, DEV) for s in specs]
    refs = [ref_decode(s, t) for s, t in zip(specs, ts)]
    streams = [torch.cuda.Stream() for _ in range(2)]
    outs = [[], []]
    torch.cuda.synchronize()
    for _ in range(6):
        for i in range(2):
            with torch.cuda.stream(streams[i]):
                t = ts[i]
                outs[i].append(M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0],
                                                        t["block_tables"], t["kv_len"], 16, strict=False,
                                                        variant="sched"))
    torch.cuda.synchronize()
    M.check_device_errors()
    for i in range(2):
        for o in outs[i]:
            close(o, refs[i], f"stream {i}")


def test_bad_sequences_get_zero_rows_and_raise():
    ctx = np.array([40, 300, 17], np.int64)
    spec = W.build_spec("bad", ctx, 14, 2, 64, 16, seed=6)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    ref = ref_decode(spec, t)
    kvl = t["kv_len"].clone()
    kvl[1] = 0
    out = torch.full_like(t["query"], 5.0)
    M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"], kvl, 16,
                             out=out, strict=False, variant="sched")
    with pytest.raises(ValueError, match="kv_len"):
        M.check_device_errors()
    assert (out[1] == 0).all()
    close(out[[0, 2]], ref[[0, 2]], "the good sequences")
