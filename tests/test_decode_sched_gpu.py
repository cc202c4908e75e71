"""The scheduled persistent decode (variant "sched", the default) and its
per-step schedule (GPU).

The schedule kernel lists every (sequence, KV head, head group) unit cut into
pieces of at most `piece` 16-token tiles, longest first; the decode kernel's
CTAs take pieces from a counter and the last piece of a split unit merges it.
These tests check the schedule itself against a CPU restatement (as sets: the
order inside a bucket is arbitrary by design), the decode against the oracle
over batch sizes from 1 to 5000 and units thousands of tiles long, the reuse
of one schedule by several layers, the write-then-decode overlap, the
backend's once-per-step build, concurrent streams, and bad sequences.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import mini_vllm_b200 as M
import oracle
from conftest import torch_to_np
from mini_vllm_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = "cuda"
MAX_PIECE, MIN_PIECE = 32, 4


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


def restated_pieces(ctx, units_per_seq, block_size, max_blocks, ctas):
    """CPU restatement of the schedule kernel's cut: {(seq, unit): [(first
    tile, tiles), ...]} and the piece length chosen."""
    def bad(c):
        return c < 1 or -(-c // block_size) > max_blocks
    total = sum(-(-c // 16) for c in ctx if not bad(c)) * units_per_seq
    piece = min(MAX_PIECE, max(MIN_PIECE, -(-total // (2 * ctas)) if total else MIN_PIECE))
    out = {}
    for s, c in enumerate(ctx):
        nt = 0 if bad(c) else -(-c // 16)
        p = 1 if bad(c) else -(-nt // piece)
        for k in range(units_per_seq):
            out[(s, k)] = [(i * nt // p, (i + 1) * nt // p - i * nt // p) for i in range(p)]
    return out, piece


def read_schedule(sched):
    ws = sched.workspace
    hdr = ws[:256].view(torch.int32).cpu().numpy()
    n = int(hdr[0])
    desc = ws[256:256 + 32 * n].view(torch.int32).cpu().numpy().reshape(n, 8)
    return hdr, desc


@pytest.mark.parametrize("num_seqs,heads", [(256, (14, 2)), (7, (14, 2)), (96, (32, 8)), (3, (40, 2))])
def test_schedule_lists_every_tile_once(num_seqs, heads):
    h, kh = heads
    d = 128 if kh == 8 else 64
    ctx = W.context_lengths(2, seed=num_seqs, num_seqs=num_seqs)
    if num_seqs == 3:
        ctx[:] = [1, 20000, 33]
    spec = W.build_spec("s", ctx, h, kh, d, 16, seed=1)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    sched = M.build_decode_schedule(t["kv_len"], h, kh, d, 16, spec.num_blocks, spec.max_blocks, torch.bfloat16)
    torch.cuda.synchronize()
    hdr, desc = read_schedule(sched)
    hg = -(-(h // kh) // 16)
    ctas = torch.cuda.get_device_properties(0).multi_processor_count
    want, piece = restated_pieces([int(c) for c in ctx], kh * hg, 16, spec.max_blocks, ctas)
    assert hdr[1] == piece and hdr[2] == 0 and hdr[3] == 0  # hand-out counters at rest
    got = {}
    sizes = []
    for i, (s, k, b0, nt, first, p, c, _flag) in enumerate(desc.tolist()):
        assert first <= i < first + p and c == ctx[s]
        assert 0 <= nt <= MAX_PIECE
        got.setdefault((s, k), []).append((b0, nt, i - first))
        sizes.append(nt)
    assert sorted(got) == sorted(want)
    for key, pieces in got.items():
        pieces.sort(key=lambda x: x[2])
        assert [(b, n) for b, n, _ in pieces] == want[key], key
    # longest first: the list's piece sizes never grow by more than the one
    # tile an even split allows between pieces of one unit
    assert all(b <= a + 1 for a, b in zip(sizes, sizes[1:]))


def test_one_schedule_serves_every_layer():
    spec = W.make_spec(2, seed=40)
    t = W.torch_tensors(spec, torch.bfloat16, DEV, num_layers=3)
    sched = M.build_decode_schedule(t["kv_len"], 14, 2, 64, 16, spec.num_blocks, spec.max_blocks, torch.bfloat16)
    for layer in range(3):
        out = M.paged_decode_attention(t["query"], t["key_caches"][layer], t["value_caches"][layer],
                                       t["block_tables"], t["kv_len"], 16, schedule=sched)
        close(out, ref_decode(spec, t, t["key_caches"][layer], t["value_caches"][layer]), f"layer {layer}")
        hdr, _ = read_schedule(sched)
        assert hdr[2] == 0 and hdr[3] == 0  # the last CTA reset the counters


@pytest.mark.parametrize("num_seqs", [1, 2, 3, 8, 37, 148, 300, 1500, 5000])
def test_batch_sizes(num_seqs):
    """From one sequence (each unit cut into 4-tile pieces across the GPU) to
    thousands (many pieces per CTA), twice in a row (the counters the first
    call left at zero)."""
    ctx = W.context_lengths(2, seed=num_seqs, num_seqs=num_seqs)
    if num_seqs <= 3:
        ctx[:] = [3000, 1, 77][:num_seqs]
    spec = W.build_spec("b", ctx, 14, 2, 64, 16, seed=num_seqs)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    ref = ref_decode(spec, t)
    for _ in range(2):
        out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                       t["kv_len"], 16, variant="sched")
        close(out, ref, f"n={num_seqs}")


@pytest.mark.parametrize("head_dim,heads,kv_heads", [(64, 14, 2), (128, 32, 8)])
def test_long_units_many_pieces(head_dim, heads, kv_heads):
    """Units thousands of tiles long: each is cut into more pieces than a warp
    has lanes, merged in rounds of 32 by the last piece to arrive."""
    ctx = np.array([40000, 5, 30001, 17], np.int64)
    spec = W.build_spec("long", ctx, heads, kv_heads, head_dim, 16, seed=41)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    sched = M.build_decode_schedule(t["kv_len"], heads, kv_heads, head_dim, 16, spec.num_blocks, spec.max_blocks,
                                    torch.bfloat16)
    _, desc = read_schedule(sched)
    assert desc[:, 5].max() > 32
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
    sched = M.build_decode_schedule(t["kv_len"], 14, 2, 64, 16, spec.num_blocks, spec.max_blocks, torch.bfloat16)
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
    o = M.paged_decode_attention(t["query"], kc, vc, t["block_tables"], t["kv_len"], 16, after_write=True)
    assert torch.equal(o, outs[0])


def test_backend_builds_the_schedule_once_per_step():
    spec, t, ref = _write_then_decode_case(34, 64)
    backend = M.AttentionBackendB200(M.ModelConfig(num_heads=14, num_kv_heads=2, head_dim=64), strict=True,
                                     overlap_after_write=True)
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
                                                        t["block_tables"], t["kv_len"], 16, strict=False))
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
                             out=out, strict=False)
    with pytest.raises(ValueError, match="kv_len"):
        M.check_device_errors()
    assert (out[1] == 0).all()
    close(out[[0, 2]], ref[[0, 2]], "the good sequences")
