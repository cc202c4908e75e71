"""The multi-GPU path's host logic on two CPU ranks over gloo (CPU only).

Each rank owns the sequences ``snake_assignment`` gives it (with its own KV
pool holding only its sequences' blocks), decodes its share, and
``gather_outputs`` all-gathers and reorders the rows.  With no GPU here the
per-rank decode is the CPU oracle — the checker standing in for the kernel;
what is under test is the sharding, the per-rank pools and the gather.
The gathered result must equal the unsharded decode bit for bit.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank: int, world: int, port: int, result_path: str):
    import sys

    repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, repo)
    import datetime

    import torch
    import torch.distributed as dist

    import oracle
    from mini_vllm_b200 import sharding
    from mini_vllm_b200 import workloads as W

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ctx = W.context_lengths(4, seed=1, num_seqs=24)
        owned = sharding.snake_assignment(ctx, world)
        mine = owned[rank]
        c = W.CONFIGS[4]
        spec = W.build_spec("shard", ctx[mine], c["num_heads"], c["num_kv_heads"], c["head_dim"],
                            c["block_size"], seed=100 + rank)
        # every rank derives the global q/K/V deterministically, then keeps its own rows/blocks
        rng = np.random.default_rng(7)
        q_all = W.f32_to_bf16_bits(rng.standard_normal((ctx.size, c["num_heads"], c["head_dim"]), dtype=np.float32))
        kc = np.zeros((spec.num_blocks, c["num_kv_heads"], c["block_size"], c["head_dim"]), np.uint16)
        vc = np.zeros_like(kc)
        for i, g in enumerate(mine.tolist()):
            r = np.random.default_rng(1000 + g)
            n = int(ctx[g])
            k = W.f32_to_bf16_bits(r.standard_normal((n, c["num_kv_heads"], c["head_dim"]), dtype=np.float32))
            v = W.f32_to_bf16_bits(r.standard_normal((n, c["num_kv_heads"], c["head_dim"]), dtype=np.float32))
            pos = np.arange(n)
            slots = spec.block_tables[i][pos // c["block_size"]] * c["block_size"] + pos % c["block_size"]
            oracle.cache_write(k, v, kc, vc, slots, c["block_size"], "bf16")
        out_local, st = oracle.decode(q_all[mine], kc, vc, spec.block_tables, spec.context_lens,
                                      c["block_size"], "bf16")
        assert (st == 0).all()
        gathered = sharding.gather_outputs(torch.from_numpy(out_local), owned, rank)
        reusable = sharding.OutputGather(owned, c["num_heads"], c["head_dim"], torch.float32,
                                         torch.device("cpu"))
        for _ in range(2):  # the buffers are reused call after call
            again = reusable(torch.from_numpy(out_local))
            assert torch.equal(again, gathered)
        # a decode that wrote straight into the send buffer (no copy)
        reusable.send_view(out_local.shape[0]).copy_(torch.from_numpy(out_local))
        assert torch.equal(reusable(reusable.send_view(out_local.shape[0])), gathered)
        if rank == 0:
            np.save(result_path, gathered.numpy())
    finally:
        dist.destroy_process_group()


def _unsharded_reference():
    import oracle
    from mini_vllm_b200 import workloads as W

    ctx = W.context_lengths(4, seed=1, num_seqs=24)
    c = W.CONFIGS[4]
    spec = W.build_spec("full", ctx, c["num_heads"], c["num_kv_heads"], c["head_dim"], c["block_size"], seed=5)
    rng = np.random.default_rng(7)
    q_all = W.f32_to_bf16_bits(rng.standard_normal((ctx.size, c["num_heads"], c["head_dim"]), dtype=np.float32))
    kc = np.zeros((spec.num_blocks, c["num_kv_heads"], c["block_size"], c["head_dim"]), np.uint16)
    vc = np.zeros_like(kc)
    for g in range(ctx.size):
        r = np.random.default_rng(1000 + g)
        n = int(ctx[g])
        k = W.f32_to_bf16_bits(r.standard_normal((n, c["num_kv_heads"], c["head_dim"]), dtype=np.float32))
        v = W.f32_to_bf16_bits(r.standard_normal((n, c["num_kv_heads"], c["head_dim"]), dtype=np.float32))
        pos = np.arange(n)
        slots = spec.block_tables[g][pos // c["block_size"]] * c["block_size"] + pos % c["block_size"]
        oracle.cache_write(k, v, kc, vc, slots, c["block_size"], "bf16")
    out, st = oracle.decode(q_all, kc, vc, spec.block_tables, spec.context_lens, c["block_size"], "bf16")
    assert (st == 0).all()
    return out


@pytest.mark.parametrize("world", [2, 3, 5])  # 5: uneven shares (5, 5, 5, 5, 4), padded in the gather
def test_sharded_decode_with_gloo_gather_matches_unsharded(tmp_path, world):
    result = str(tmp_path / "gathered.npy")
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, result)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    gathered = np.load(result)
    assert np.array_equal(gathered, _unsharded_reference())

