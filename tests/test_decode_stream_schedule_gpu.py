"""The stream decode (variant "stream") reading a per-step schedule (GPU).

A model step's layers share kv_len and the block tables, so the stream
kernel's set-up — the tile prefix of every sequence, the pool row of every KV
tile of the stream and each warp's range — is built once per step
(mvb_paged_decode_schedule with MVB_DECODE_STREAM) and every layer's decode
starts from it (MVB_DECODE_SCHEDULE_READY).  The schedule cuts the cost-aware
split (a warp's tiles plus one tile's cost per unit it enters) where it
applies, the kernel without a schedule the equal split, so the two forms agree
bit for bit only where the cost split does not apply; both must match the
oracle (csrc/oracle.c, a restatement of paged_attention_gpu.py:464-575) within
the decode bound 2e-3 + 1e-2 |ref|, and each is deterministic.  Cases: the benchmark's config-2 batch,
GQA 14/2 at head_dim 64 and 32/8 at 128, batches of 1 to 1500, one schedule
over several layers, the write-then-decode overlap, the backend's
once-per-step build, left-out sequences and bad block ids, and a plan without a
per-step set-up.
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


def _schedule(t, spec, h, kh, d, **kw):
    return M.build_decode_schedule(t["kv_len"], t["block_tables"], h, kh, d, spec.block_size, spec.num_blocks,
                                   torch.bfloat16, variant="stream", **kw)


def _decode(t, spec, layer=0, **kw):
    return M.paged_decode_attention(t["query"], t["key_caches"][layer], t["value_caches"][layer],
                                    t["block_tables"], t["kv_len"], spec.block_size, variant="stream", **kw)


@pytest.mark.parametrize("num_seqs,heads", [(256, (14, 2)), (96, (32, 8)), (7, (14, 2)), (1, (14, 2)),
                                            (1500, (14, 2)), (3, (40, 2))])
def test_schedule_matches_the_oracle_and_is_deterministic(num_seqs, heads):
    h, kh = heads
    d = 128 if kh == 8 else 64
    ctx = W.context_lengths(2, seed=num_seqs, num_seqs=num_seqs)
    if num_seqs == 1:
        ctx[:] = [20000]  # one unit cut across every warp of the GPU
    if num_seqs == 3:
        ctx[:] = [1, 5000, 33]  # GQA 20: two head groups per KV head
    spec = W.build_spec("s", ctx, h, kh, d, 16, seed=num_seqs + 1)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    sched = _schedule(t, spec, h, kh, d)
    assert sched.variant == "stream" and sched.workspace is not None
    inline = _decode(t, spec)
    ready = _decode(t, spec, schedule=sched)
    M.check_device_errors()
    ref = ref_decode(spec, t)
    close(ready, ref, f"n={num_seqs} GQA {h}/{kh} D={d}, with the schedule")
    close(inline, ref, f"n={num_seqs} GQA {h}/{kh} D={d}, without")
    assert torch.equal(ready, _decode(t, spec, schedule=sched)), "a fixed work split: the same bits every time"


def test_one_schedule_serves_every_layer():
    spec = W.make_spec(2, seed=60)
    L = 4
    t = W.torch_tensors(spec, torch.bfloat16, DEV, num_layers=L)
    sched = _schedule(t, spec, 14, 2, 64)
    first = []
    for rep in range(2):
        for layer in range(L):
            out = _decode(t, spec, layer, schedule=sched)
            ref = ref_decode(spec, t, t["key_caches"][layer], t["value_caches"][layer])
            close(out, ref, f"rep {rep} layer {layer}")
            if rep == 0:
                first.append(out)
            else:
                assert torch.equal(out, first[layer])


def test_auto_takes_the_schedule_variant():
    """variant "auto" with a stream schedule runs the stream kernel from it;
    an explicit other kernel with that schedule is refused."""
    spec = W.make_spec(2, seed=61)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    sched = M.build_decode_schedule(t["kv_len"], t["block_tables"], 14, 2, 64, 16, spec.num_blocks, torch.bfloat16)
    assert sched.variant == "stream"  # AUTO's kernel at config 2
    out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                   t["kv_len"], 16, schedule=sched)
    assert torch.equal(out, _decode(t, spec, schedule=sched))
    with pytest.raises(Exception, match="schedule"):
        M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                 t["kv_len"], 16, schedule=sched, variant="sched")


@pytest.mark.parametrize("num_seqs", [256, 5])
def test_write_then_decode_with_a_schedule(num_seqs):
    """The bench's step order: schedule, then per layer the KV write and the
    decode with its inputs read while the write runs.  The new tokens
    dominate attention (K = 4, V = 3), so a decode that read the cache before
    the write landed would be far off."""
    spec = W.make_spec(2, seed=62, num_seqs=num_seqs)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    t["new_key"].fill_(4.0)
    t["new_value"].fill_(3.0)
    kc, vc = torch_to_np(t["key_caches"][0], "bf16"), torch_to_np(t["value_caches"][0], "bf16")
    oracle.cache_write(torch_to_np(t["new_key"], "bf16"), torch_to_np(t["new_value"], "bf16"), kc, vc,
                       spec.slot_mapping, 16, "bf16")
    ref, st = oracle.decode(torch_to_np(t["query"], "bf16"), kc, vc, spec.block_tables, spec.context_lens, 16,
                            "bf16")
    assert (st == 0).all()
    sched = _schedule(t, spec, 14, 2, 64)
    outs = []
    for _ in range(3):
        kcg, vcg = t["key_caches"][0].clone(), t["value_caches"][0].clone()
        M.paged_cache_write(t["new_key"], t["new_value"], kcg, vcg, t["slot_mapping"], 16, strict=False,
                            check_duplicates=False)
        o = M.paged_decode_attention(t["query"], kcg, vcg, t["block_tables"], t["kv_len"], 16, strict=False,
                                     after_write=True, schedule=sched)
        M.check_device_errors()
        close(o, ref, "after_write + schedule")
        outs.append(o)
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[1], outs[2])
    # the schedule built right after the write (after_write: its inputs are read while the write runs)
    kcg, vcg = t["key_caches"][0].clone(), t["value_caches"][0].clone()
    M.paged_cache_write(t["new_key"], t["new_value"], kcg, vcg, t["slot_mapping"], 16)
    sched2 = _schedule(t, spec, 14, 2, 64, after_write=True, schedule=sched)
    o = M.paged_decode_attention(t["query"], kcg, vcg, t["block_tables"], t["kv_len"], 16, schedule=sched2)
    assert torch.equal(o, outs[0])


def test_backend_builds_the_stream_schedule_once_per_step():
    spec = W.make_spec(2, seed=63, num_seqs=64)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    backend = M.AttentionBackendB200(M.ModelConfig(num_heads=14, num_kv_heads=2, head_dim=64), strict=True,
                                     overlap_after_write=True)
    L = 3
    kcs = [t["key_caches"][0].clone() for _ in range(L)]
    vcs = [t["value_caches"][0].clone() for _ in range(L)]
    pool = M.KVCachePool(kcs, vcs, spec.num_blocks, 16, L, 2, 64, torch.device(DEV), torch.bfloat16)
    backend._pool = pool
    kc, vc = torch_to_np(t["key_caches"][0], "bf16"), torch_to_np(t["value_caches"][0], "bf16")
    oracle.cache_write(torch_to_np(t["new_key"], "bf16"), torch_to_np(t["new_value"], "bf16"), kc, vc,
                       spec.slot_mapping, 16, "bf16")
    ref, st = oracle.decode(torch_to_np(t["query"], "bf16"), kc, vc, spec.block_tables, spec.context_lens, 16,
                            "bf16")
    assert (st == 0).all()

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
            assert backend._schedule.variant == "stream"
            if first is None:
                first = o
            assert torch.equal(o, first)


def test_left_out_sequences_and_bad_block_ids():
    """kv_len 0, a table too short for kv_len and an out-of-range block id: the
    schedule build flags them; every decode from the schedule flags them again,
    zeroes the rows of the left-out sequences and gives the inline bits (a
    batch with left-out sequences is cut with the equal split)."""
    ctx = np.array([40, 300, 17, 700, 90], np.int64)
    spec = W.build_spec("bad", ctx, 14, 2, 64, 16, seed=7)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    ref = ref_decode(spec, t)
    kvl = t["kv_len"].clone()
    kvl[1] = 0
    kvl[3] = spec.max_blocks * 16 + 1  # past the table
    bt = t["block_tables"].clone()
    bt[4, 2] = spec.num_blocks + 3  # tile 2 of sequence 4: no such block
    sched = M.build_decode_schedule(kvl, bt, 14, 2, 64, 16, spec.num_blocks, torch.bfloat16, variant="stream",
                                    strict=False)
    with pytest.raises((ValueError, IndexError)):
        M.check_device_errors()
    outs = []
    for sc in (sched, None):
        out = torch.full_like(t["query"], 5.0)
        M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], bt, kvl, 16, out=out,
                                 strict=False, variant="stream", schedule=sc)
        with pytest.raises((ValueError, IndexError)):
            M.check_device_errors()
        assert (out[1] == 0).all() and (out[3] == 0).all()
        close(out[[0, 2]], ref[[0, 2]], "the good sequences")
        outs.append(out)
    assert torch.equal(outs[0], outs[1])
    # the same error bits from both forms: kv_len, table short, block id
    from mini_vllm_b200.attention import paged_attention_b200 as PA

    errs = []
    for sc in (sched, None):
        M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], bt, kvl, 16, strict=False,
                                 variant="stream", schedule=sc)
        torch.cuda.synchronize()
        errs.append(PA._take_flags(PA._state(torch.device(DEV, 0))))
    from mini_vllm_b200 import _native

    assert errs[0] == errs[1] == _native.DEV_KV_LEN | _native.DEV_TABLE_SHORT | _native.DEV_BLOCK_ID


def test_fp32_plans_no_per_step_set_up():
    """fp32 runs the CUDA-core kernel, which has no per-step set-up: the
    schedule is empty and the decode runs as without one."""
    spec = W.make_spec(2, seed=64, num_seqs=12)
    t = W.torch_tensors(spec, torch.float32, DEV)
    sched = M.build_decode_schedule(t["kv_len"], t["block_tables"], 14, 2, 64, 16, spec.num_blocks, torch.float32)
    assert sched.variant is None and sched.workspace is None
    a = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                 t["kv_len"], 16, schedule=sched)
    b = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                 t["kv_len"], 16)
    assert torch.equal(a, b)
