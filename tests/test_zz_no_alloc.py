"""The allocation-free decode entry point against the workspace one (GPU).

mvb_paged_decode_noalloc serves callers that cannot allocate device memory at
decode time — a server that hands all free HBM to the KV pool at start-up, or
a host binding with no device allocator — by keeping the split-K partial
states in a fixed array inside the library.  It must give the same output as
mvb_paged_decode with a caller workspace, call after call (the array is
shared and keeps the previous call's contents), and refuse shapes whose
partials do not fit the array.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import mini_vllm_b200 as M
from mini_vllm_b200 import _native
from mini_vllm_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _noalloc(t, spec, out, err, variant, partition_tokens):
    q = t["query"]
    kc, vc = t["key_caches"][0], t["value_caches"][0]
    bt = t["block_tables"]
    return _native.lib().mvb_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), vc.data_ptr(),
        bt.data_ptr(), bt.stride(0), bt.shape[1], t["kv_len"].data_ptr(),
        out.data_ptr(), out.stride(0), out.stride(1),
        spec.num_seqs, spec.num_heads, spec.num_kv_heads, spec.head_dim, spec.block_size,
        spec.num_blocks, spec.head_dim ** -0.5, _native.DTYPE_BF16, variant, partition_tokens,
        err.data_ptr(), torch.cuda.current_stream(DEV).cuda_stream)


def _close(a: torch.Tensor, b: torch.Tensor):
    # the tolerance the decode parity tests use for bf16: 2e-3 + 1e-2 * |ref|
    x, y = a.float(), b.float()
    assert torch.isfinite(x).all()
    assert ((x - y).abs() <= 2e-3 + 1e-2 * y.abs()).all()


@pytest.mark.parametrize("variant,partition_tokens,num_seqs", [
    (_native.DECODE_MMA, 512, 256),   # split-K on the tensor cores, 1-4 partitions per sequence
    (_native.DECODE_AUTO, 256, 64),   # AUTO resolves to the split-K tensor-core kernel here
    (_native.DECODE_FMA, 512, 48),    # split-K on CUDA cores
])
def test_noalloc_matches_workspace_entry_point_twice(variant, partition_tokens, num_seqs):
    spec = W.make_spec(2, seed=17, num_seqs=num_seqs)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    name = {_native.DECODE_MMA: "mma", _native.DECODE_AUTO: "mma", _native.DECODE_FMA: "fma"}[variant]
    plan = M.decode_plan(spec.num_seqs, spec.num_heads, spec.num_kv_heads, spec.head_dim, spec.block_size,
                         spec.num_blocks, spec.max_blocks, torch.bfloat16, name, partition_tokens)
    assert plan["num_partitions"] > 1  # the scratch array is really used
    ref = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                   t["kv_len"], spec.block_size, variant=name,
                                   partition_tokens=partition_tokens)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.full_like(ref, float("nan"))
    st = _noalloc(t, spec, out, err, variant, partition_tokens)
    assert st == _native.OK, _native.status_string(st)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    _close(out, ref)
    assert torch.equal(out, ref)  # same kernels, same partitions: the same bits
    # The second call finds the first call's partials in the array.  Other
    # inputs with shorter contexts (fewer partitions per sequence) show that
    # every partial it reads, it wrote first.
    ctx2 = np.maximum(1, W.make_spec(2, seed=117, num_seqs=num_seqs).context_lens // 3)
    spec2 = W.build_spec("short", ctx2, spec.num_heads, spec.num_kv_heads, spec.head_dim, spec.block_size,
                         seed=117)
    t2 = W.torch_tensors(spec2, torch.bfloat16, DEV)
    ref2 = M.paged_decode_attention(t2["query"], t2["key_caches"][0], t2["value_caches"][0], t2["block_tables"],
                                    t2["kv_len"], spec.block_size, variant=name, partition_tokens=partition_tokens)
    out2 = torch.full_like(ref2, float("nan"))
    st = _noalloc(t2, spec2, out2, err, variant, partition_tokens)
    assert st == _native.OK, _native.status_string(st)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    _close(out2, ref2)
    assert torch.equal(out2, ref2)


def test_noalloc_rejects_shapes_beyond_its_array():
    spec = W.make_spec(2, seed=18)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    # 16-token partitions: 256 x 14 x 128 partials x (64 + 2) floats is far above 16 MiB
    plan = M.decode_plan(spec.num_seqs, 14, 2, 64, 16, spec.num_blocks, spec.max_blocks, torch.bfloat16,
                         "mma", 16)
    assert plan["workspace_bytes"] > 16 << 20
    out = torch.empty_like(t["query"])
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    assert _noalloc(t, spec, out, err, _native.DECODE_MMA, 16) == _native.ERR_WORKSPACE
    assert _noalloc(t, spec, out, err, _native.DECODE_STREAM, 0) == _native.ERR_VARIANT


def test_noalloc_handles_unsplit_and_small_batches():
    ctx = np.array([1, 17, 300], np.int64)
    spec = W.build_spec("s", ctx, 14, 2, 64, 16, seed=3)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    ref = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                   t["kv_len"], 16, variant="mma")
    out = torch.empty_like(ref)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    assert _noalloc(t, spec, out, err, _native.DECODE_AUTO, 0) == _native.OK
    torch.cuda.synchronize()
    _close(out, ref)
