"""Host-side logic of the plug-in, without a GPU (CPU only).

Covers the factory and the no-silent-fallback contract (the reference's
test_no_silent_fallback.py), the KV pool (test_kv_cache_pool.py), argument
validation of the free functions, the workload generator and the sharding
assignment.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import mini_vllm_b200 as M
from mini_vllm_b200 import sharding
from mini_vllm_b200 import workloads as W
from mini_vllm_b200.attention import validate_block_size
from mini_vllm_b200.cache import MIN_BLOCKS, KVCachePool, compute_num_gpu_blocks


def cfg(**kw):
    base = dict(num_layers=1, hidden_size=256, num_heads=4, num_kv_heads=2, head_dim=64,
                dtype=torch.float16)
    base.update(kw)
    return M.ModelConfig(**base)


# --------------------------------------------------------------------------- factory
def test_factory_unknown_backend_raises_value_error():
    with pytest.raises(ValueError, match="Unknown"):
        M.AttentionBackend.create(cfg(), backend="nonexistent")


@pytest.mark.parametrize("name", ["triton", "reference", "ref"])
def test_factory_has_no_other_backends(name):
    with pytest.raises(ValueError, match="Unknown"):
        M.AttentionBackend.create(cfg(), backend=name)


def test_unsupported_head_dim_raises_runtime_error():
    with pytest.raises(RuntimeError, match="head_dim"):
        M.AttentionBackendB200(cfg(head_dim=96))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-CUDA path")
def test_no_cuda_raises_runtime_error_not_fallback():
    with pytest.raises(RuntimeError, match="requires CUDA"):
        M.AttentionBackend.create(cfg(), backend="b200")


@pytest.mark.parametrize("bs", [0, -4, 3, 12, 24])
def test_block_size_must_be_power_of_two(bs):
    with pytest.raises(RuntimeError, match="block_size"):
        validate_block_size(bs)


@pytest.mark.parametrize("bs", [1, 2, 4, 8, 16, 32, 64, 128, 256])
def test_block_size_powers_of_two_accepted(bs):
    validate_block_size(bs)


def test_argument_error_is_both_assertion_and_value_error():
    assert issubclass(M.ArgumentError, AssertionError) and issubclass(M.ArgumentError, ValueError)


# --------------------------------------------------------------------------- free-function validation
def _kv(t=2, kh=2, d=8, dtype=torch.float16):
    return torch.zeros(t, kh, d, dtype=dtype), torch.zeros(t, kh, d, dtype=dtype)


@pytest.mark.parametrize("mutate,match", [
    (lambda a: a.update(value=torch.zeros(2, 2, 9, dtype=torch.float16)), r"key .* != value"),
    (lambda a: a.update(value_cache=torch.zeros(2, 2, 4, 8, dtype=torch.float16)), "cache shape"),
    (lambda a: a.update(slot_mapping=torch.tensor([0])), "slot_mapping length"),
    (lambda a: a.update(key=torch.zeros(2, 4, 8, dtype=torch.float16),
                        value=torch.zeros(2, 4, 8, dtype=torch.float16)), "num_kv_heads"),
    (lambda a: a.update(key=torch.zeros(2, 2, 16, dtype=torch.float16),
                        value=torch.zeros(2, 2, 16, dtype=torch.float16)), "head_dim"),
    (lambda a: a.update(block_size=8), "block_size"),
    (lambda a: a.update(block_size=0), "block_size must be > 0"),
    (lambda a: a.update(key=torch.zeros(2, 2, 8), value=torch.zeros(2, 2, 8)), "dtype"),
    (lambda a: None, "cuda"),
])
def test_cache_write_validation_messages(mutate, match):
    k, v = _kv()
    args = dict(key=k, value=v, key_cache=torch.zeros(4, 2, 4, 8, dtype=torch.float16),
                value_cache=torch.zeros(4, 2, 4, 8, dtype=torch.float16),
                slot_mapping=torch.tensor([0, 1]), block_size=4)
    mutate(args)
    with pytest.raises(ValueError, match=match):
        M.paged_cache_write(**args)


@pytest.mark.parametrize("mutate,match", [
    (lambda a: a.update(query=torch.zeros(1, 4, 96, dtype=torch.bfloat16),
                        key_cache=torch.zeros(4, 2, 16, 96, dtype=torch.bfloat16),
                        value_cache=torch.zeros(4, 2, 16, 96, dtype=torch.bfloat16)), "head_dim"),
    (lambda a: a.update(block_size=12), "power of 2"),
    (lambda a: a.update(query=torch.zeros(1, 3, 64, dtype=torch.bfloat16)), "divisible"),
    (lambda a: a.update(query=torch.zeros(1, 4, 64, dtype=torch.float64)), "dtype"),
    (lambda a: a.update(block_table=torch.zeros(2, 1, dtype=torch.long)), "block_table rows"),
    (lambda a: a.update(kv_len_after=torch.ones(2, dtype=torch.int32)), "kv_len_after shape"),
    (lambda a: None, "cuda"),
])
def test_decode_validation_messages(mutate, match):
    args = dict(query=torch.zeros(1, 4, 64, dtype=torch.bfloat16),
                key_cache=torch.zeros(4, 2, 16, 64, dtype=torch.bfloat16),
                value_cache=torch.zeros(4, 2, 16, 64, dtype=torch.bfloat16),
                block_table=torch.zeros(1, 1, dtype=torch.long),
                kv_len_after=torch.ones(1, dtype=torch.int32), block_size=16)
    mutate(args)
    with pytest.raises(AssertionError, match=match):
        M.paged_decode_attention(**args)


# --------------------------------------------------------------------------- pool (test_kv_cache_pool.py)
def test_pool_allocate_shapes_and_accessors():
    pool = KVCachePool.allocate(2, 8, 4, 4, 128, dtype=torch.float16, device=torch.device("cpu"))
    assert (pool.num_layers, pool.num_blocks, pool.block_size, pool.num_kv_heads, pool.head_dim) == (2, 8, 4, 4, 128)
    assert len(pool.key_caches) == len(pool.value_caches) == 2
    for l in range(2):
        assert pool.key_caches[l].shape == pool.value_caches[l].shape == (8, 4, 4, 128)
        assert pool.get_key_cache(l) is pool.key_caches[l]
        assert pool.get_value_cache(l) is pool.value_caches[l]
        assert pool.key_caches[l].is_contiguous()


@pytest.mark.parametrize("args,name", [
    ((1, 0, 4, 2, 64), "num_blocks"), ((0, 8, 4, 2, 64), "num_layers"), ((1, 8, 0, 2, 64), "block_size"),
    ((1, 8, 4, 0, 64), "num_kv_heads"), ((1, 8, 4, 2, 0), "head_dim"),
])
def test_pool_invalid_params(args, name):
    with pytest.raises(ValueError, match=name):
        KVCachePool.allocate(*args)


def test_pool_reset_and_byte_properties():
    pool = KVCachePool.allocate(3, 8, 4, 2, 64, dtype=torch.bfloat16, device=torch.device("cpu"))
    pool.key_caches[1].fill_(3)
    pool.reset()
    assert all((k == 0).all() and (v == 0).all() for k, v in zip(pool.key_caches, pool.value_caches))
    assert pool.total_slots == 32
    assert pool.bytes_per_block_per_layer == 2 * 2 * 4 * 64 * 2
    assert pool.bytes_per_block_total == 3 * pool.bytes_per_block_per_layer
    assert pool.total_bytes == 8 * pool.bytes_per_block_total


def test_compute_num_gpu_blocks_rules():
    assert compute_num_gpu_blocks(2, 2, 64, 16, num_gpu_blocks_override=100) == 100
    with pytest.raises(RuntimeError, match="minimum"):
        compute_num_gpu_blocks(2, 2, 64, 16, num_gpu_blocks_override=MIN_BLOCKS - 1)
    with pytest.raises(ValueError, match="gpu_memory_utilization"):
        compute_num_gpu_blocks(2, 2, 64, 16, gpu_memory_utilization=0.0)
    assert compute_num_gpu_blocks(2, 2, 64, 16, device=torch.device("cpu")) == MIN_BLOCKS


# --------------------------------------------------------------------------- workloads
@pytest.mark.parametrize("config", [1, 2, 3, 4])
def test_workload_tables_are_disjoint_and_cover_context(config):
    spec = W.make_spec(config, seed=3, num_seqs=64 if config == 4 else None)
    bs = spec.block_size
    need = (spec.context_lens + bs - 1) // bs
    used = []
    for s in range(spec.num_seqs):
        row = spec.block_tables[s]
        assert (row[: need[s]] >= 0).all() and (row[need[s]:] == -1).all()
        used.extend(row[: need[s]].tolist())
    assert len(used) == len(set(used)) and max(used) < spec.num_blocks
    # the write slot is the last context position of each sequence
    last = spec.context_lens - 1
    exp = spec.block_tables[np.arange(spec.num_seqs), last // bs] * bs + last % bs
    assert np.array_equal(spec.slot_mapping, exp)


def test_workload_config_shapes():
    s1 = W.make_spec(1)
    assert (s1.num_seqs, s1.num_heads, s1.num_kv_heads, s1.head_dim, s1.num_blocks) == (8, 14, 2, 64, 512)
    assert s1.context_lens.min() >= 1 and s1.context_lens.max() <= 512
    s2 = W.make_spec(2)
    assert s2.num_seqs == 256 and s2.context_lens.min() >= 128 and s2.context_lens.max() <= 2048
    need = int(((s2.context_lens + 15) // 16).sum())
    assert s2.num_blocks == int(np.ceil(1.1 * need))
    s3 = W.make_spec(3)
    assert (s3.context_lens == 32768).all() and s3.num_seqs == 32
    ctx4 = W.context_lengths(4)
    assert ctx4.size == 1024 and ctx4.min() >= 16 and ctx4.max() <= 8192


def test_workload_is_deterministic_and_bf16_rounding_is_rne():
    a, b = W.make_spec(2, seed=9), W.make_spec(2, seed=9)
    assert np.array_equal(a.block_tables, b.block_tables)
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5e-8, 3.0e38], np.float32)
    got = (W.f32_to_bf16_bits(x).astype(np.uint32) << 16).view(np.float32)
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    assert np.array_equal(got, want)


def test_decode_bytes_formula():
    spec = W.build_spec("t", np.array([16, 17]), 14, 2, 64, 16)
    kv = (16 + 17) * 2 * 2 * 64 * 2
    qo = 2 * 2 * 14 * 64 * 2
    assert spec.decode_bytes(2) == kv + qo + 8 * 3 + 4 * 2


# --------------------------------------------------------------------------- sharding
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_snake_assignment_is_a_balanced_partition(world):
    ctx = W.context_lengths(4, seed=0)
    owned = sharding.snake_assignment(ctx, world)
    allidx = np.concatenate(owned)
    assert np.array_equal(np.sort(allidx), np.arange(ctx.size))
    counts = [o.size for o in owned]
    assert max(counts) - min(counts) <= 1
    toks = [int(ctx[o].sum()) for o in owned]
    assert max(toks) / (sum(toks) / world) < 1.02


def test_snake_assignment_uneven_batch():
    owned = sharding.snake_assignment(np.array([5, 1, 9, 3, 7]), 2)
    assert sorted(np.concatenate(owned).tolist()) == [0, 1, 2, 3, 4]
    assert sorted(o.size for o in owned) == [2, 3]


def test_gather_host_checks_without_gpu():
    """The gather's host-side contract: a table too short for the requested
    tokens raises IndexError (gather_paged_kv, cache_read.py:62-67) and host
    caches are rejected before any device work."""
    kc = torch.zeros(4, 2, 16, 64, dtype=torch.bfloat16)
    with pytest.raises(IndexError, match="insufficient to cover 40 tokens"):
        M.gather_paged_kv(kc, kc, [0, 1], 40, 16)
    with pytest.raises(M.ArgumentError, match="one CUDA device"):
        M.paged_gather(kc, kc, torch.zeros(1, 2, dtype=torch.int64), [0], [4], 16)
    with pytest.raises(M.ArgumentError, match="mismatch"):
        M.paged_gather(kc, kc[:2], torch.zeros(1, 2, dtype=torch.int64), [0], [4], 16)


def test_staging_rejects_bad_arguments_before_any_cuda_call():
    """mini_vllm_b200.staging checks its tensors on the host: two host tensors
    raise ValueError before the binding is reached."""
    with pytest.raises(ValueError, match="exactly one"):
        M.staging.stream_copy(torch.zeros(4), torch.zeros(4), None)
