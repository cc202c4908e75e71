"""KV-cache write kernel vs the oracle / reference golden vectors — bit-exact (GPU).

Ports the reference's TestCacheWrite (test_paged_attention_gpu.py:159-207) and
test_cache_write.py scenarios onto the CUDA kernel, plus BASELINE-size writes.
The bar is bit equality of the whole pool (written and untouched rows).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import make_golden as MG
import mini_vllm_b200 as M
import oracle
from conftest import np_to_torch, torch_to_np
from mini_vllm_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _dupes(slots) -> bool:
    s = [x for x in slots if x != -1]
    return len(s) != len(set(s))


@pytest.mark.parametrize("kind", ["write", "write_spec"])
def test_golden_writes_bit_exact(golden, kind):
    cases, arrays = golden
    for c in [c for c in cases if c["kind"] == kind]:
        x = MG.write_inputs(c) if kind == "write" else MG.write_spec_inputs(c)
        bs = c.get("block_size") or x["block_size"]
        dt = c["dtype"]
        kc, vc = np_to_torch(x["kc0"], dt, DEV), np_to_torch(x["vc0"], dt, DEV)
        key, value = np_to_torch(x["key"], dt, DEV), np_to_torch(x["value"], dt, DEV)
        slots = torch.from_numpy(x["slots"]).to(DEV)
        if _dupes(x["slots"].tolist()):
            # the reference's Triton entry forbids duplicates (AssertionError)
            with pytest.raises(AssertionError, match="Duplicate"):
                M.paged_cache_write(key, value, kc, vc, slots, bs)
            continue
        if c.get("error"):
            with pytest.raises(IndexError, match="out of range"):
                M.paged_cache_write(key, value, kc, vc, slots, bs)
            continue
        M.paged_cache_write(key, value, kc, vc, slots, bs)
        torch.cuda.synchronize()
        assert MG.sha(torch_to_np(kc, dt), torch_to_np(vc, dt)) == c["result_sha256"], c["name"]


def _kv_ramp(shape, base):
    """The reference GPU tests' deterministic input: flat[i] = base + i (fp16)."""
    n = int(np.prod(shape))
    return (base + torch.arange(n, dtype=torch.float32, device=DEV)).to(torch.float16).view(shape)


@pytest.mark.parametrize("slots,bs,nb", [
    ([5], 16, 64),                   # test_single_token
    ([0, 17, 33, 50, 99], 16, 32),   # test_multi_token_noncontiguous
    ([7, 8], 4, 8),                  # test_block_boundary
    ([0, -1, 15], 16, 64),           # test_slot_negative_one_skips
])
def test_reference_gpu_write_cases(slots, bs, nb):
    t = len(slots)
    key, value = _kv_ramp((t, 2, 64), 10.0), _kv_ramp((t, 2, 64), 100.0)
    kc = torch.randn(nb, 2, bs, 64, device=DEV).half()
    vc = torch.randn(nb, 2, bs, 64, device=DEV).half()
    kc_ref, vc_ref = torch_to_np(kc, "f16"), torch_to_np(vc, "f16")
    oracle.cache_write(torch_to_np(key, "f16"), torch_to_np(value, "f16"), kc_ref, vc_ref,
                       np.asarray(slots), bs, "f16")
    M.paged_cache_write(key, value, kc, vc, torch.tensor(slots, device=DEV), bs)
    assert np.array_equal(torch_to_np(kc, "f16"), kc_ref)
    assert np.array_equal(torch_to_np(vc, "f16"), vc_ref)


def test_duplicate_slot_raises():
    kc = torch.empty(64, 2, 16, 64, device=DEV, dtype=torch.float16)
    vc = torch.empty_like(kc)
    key, value = _kv_ramp((2, 2, 64), 10.0), _kv_ramp((2, 2, 64), 500.0)
    with pytest.raises(AssertionError, match="Duplicate"):
        M.triton_cache_write(key, value, kc, vc, torch.tensor([5, 5], device=DEV), 16)


def test_same_slots_in_consecutive_calls_are_not_duplicates():
    kc = torch.zeros(16, 2, 16, 64, device=DEV, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    for i in range(5):
        key = torch.full((3, 2, 64), float(i), device=DEV, dtype=torch.bfloat16)
        M.paged_cache_write(key, -key, kc, vc, torch.tensor([1, 40, 255], device=DEV), 16)
    assert (kc[2, :, 8] == 4).all() and (vc[2, :, 8] == -4).all()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_strided_value_view_of_fused_qkv(dtype):
    """V as a strided view of a fused QKV GEMM output (qkv_proj.py:139-143)."""
    T, H, KH, D, BS, NB = 37, 14, 2, 64, 16, 64
    qkv = torch.randn(T, (H + 2 * KH) * D, device=DEV).to(dtype)
    heads = qkv.view(T, H + 2 * KH, D)
    k, v = heads[:, H:H + KH], heads[:, H + KH:]
    assert not v.is_contiguous()
    slots = torch.randperm(NB * BS, device=DEV)[:T]
    kc = torch.randn(NB, KH, BS, D, device=DEV).to(dtype)
    vc = torch.randn(NB, KH, BS, D, device=DEV).to(dtype)
    kc2, vc2 = kc.clone(), vc.clone()
    M.paged_cache_write(k, v, kc, vc, slots, BS)
    M.paged_cache_write(k.contiguous(), v.contiguous(), kc2, vc2, slots, BS)
    assert torch.equal(kc, kc2) and torch.equal(vc, vc2)
    blk, off = slots // BS, slots % BS
    assert torch.equal(kc[blk, :, off, :], k) and torch.equal(vc[blk, :, off, :], v)


@pytest.mark.parametrize("config,dtype,num_seqs", [(2, "bf16", None), (4, "bf16", 128), (1, "f32", None)])
def test_baseline_size_write_bit_exact(config, dtype, num_seqs):
    spec = W.make_spec(config, seed=11, num_seqs=num_seqs)
    tdt = {"bf16": torch.bfloat16, "f32": torch.float32}[dtype]
    t = W.torch_tensors(spec, tdt, DEV)
    kc, vc = t["key_caches"][0], t["value_caches"][0]
    kc_ref, vc_ref = torch_to_np(kc, dtype), torch_to_np(vc, dtype)
    oracle.cache_write(torch_to_np(t["new_key"], dtype), torch_to_np(t["new_value"], dtype), kc_ref, vc_ref,
                       spec.slot_mapping, spec.block_size, dtype)
    M.paged_cache_write(t["new_key"], t["new_value"], kc, vc, t["slot_mapping"], spec.block_size)
    assert np.array_equal(torch_to_np(kc, dtype), kc_ref)
    assert np.array_equal(torch_to_np(vc, dtype), vc_ref)


def test_prefill_sized_write_many_tokens():
    """A large prefill chunk: every slot of 300 blocks rewritten, shuffled."""
    NB, KH, BS, D = 300, 8, 16, 128
    T = NB * BS
    slots = torch.randperm(T, device=DEV)
    key = torch.randn(T, KH, D, device=DEV, dtype=torch.bfloat16)
    value = torch.randn(T, KH, D, device=DEV, dtype=torch.bfloat16)
    kc = torch.empty(NB, KH, BS, D, device=DEV, dtype=torch.bfloat16)
    vc = torch.empty_like(kc)
    M.paged_cache_write(key, value, kc, vc, slots, BS)
    blk, off = slots // BS, slots % BS
    assert torch.equal(kc[blk, :, off, :], key) and torch.equal(vc[blk, :, off, :], value)


def test_out_of_range_slot_raises_index_error_and_names_it():
    kc = torch.zeros(4, 2, 4, 64, device=DEV, dtype=torch.float16)
    vc = torch.zeros_like(kc)
    key = torch.ones(3, 2, 64, device=DEV, dtype=torch.float16)
    with pytest.raises(IndexError, match=r"slot_mapping\[1\] = 16 out of range \[0, 16\)"):
        M.paged_cache_write(key, key, kc, vc, torch.tensor([0, 16, 3], device=DEV), 4)
    # the valid tokens were still written (the kernel skips only the bad one)
    assert (kc[0, :, 0] == 1).all() and (kc[0, :, 3] == 1).all()


def test_non_strict_defers_errors_until_checked():
    kc = torch.zeros(4, 2, 4, 64, device=DEV, dtype=torch.float16)
    key = torch.ones(1, 2, 64, device=DEV, dtype=torch.float16)
    M.paged_cache_write(key, key, kc, kc.clone(), torch.tensor([-5], device=DEV), 4, strict=False)
    with pytest.raises(IndexError):
        M.check_device_errors(torch.device(DEV))
    M.check_device_errors(torch.device(DEV))  # consumed: nothing left


def test_empty_write_and_cpu_inputs_rejected():
    kc = torch.zeros(4, 2, 4, 64, device=DEV, dtype=torch.float16)
    e = torch.empty(0, 2, 64, device=DEV, dtype=torch.float16)
    M.paged_cache_write(e, e, kc, kc.clone(), torch.empty(0, dtype=torch.long, device=DEV), 4)
    with pytest.raises(AssertionError, match="device"):
        M.paged_cache_write(e.cpu(), e.cpu(), kc, kc, torch.empty(0, dtype=torch.long), 4)
