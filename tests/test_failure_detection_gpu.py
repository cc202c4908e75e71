"""A pipeline wait that runs out is reported, not hung or trapped (GPU).

The decode kernels' waits on their TMA stages are bounded.  The test hook
mvb_test_decode_wait_timeout leaves the load of one tile unissued — a stage
that nothing completes — with a short bound: the wait on it runs out, the
device error word gets MVB_DEV_TIMEOUT, the host maps it to a RuntimeError,
and the next decode on the same context is correct.  In the scheduled kernel
the timeout aborts the whole CTA (every other role's wait sees the abort
flag) while the other CTAs finish.  No trap, no fault, no unbounded wait: the
hold ends after a few thousand try-waits.
"""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import mini_vllm_b200 as M
import oracle
from conftest import torch_to_np
from mini_vllm_b200 import _native
from mini_vllm_b200 import workloads as W

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


@pytest.mark.parametrize("variant", ["stream", "sched"])
def test_wait_that_runs_out_is_reported_and_the_context_stays_usable(variant):
    spec = W.make_spec(2, seed=13, num_seqs=128)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    q, kc, vc, bt, kvl = t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"], t["kv_len"]
    plan = M.decode_plan(spec.num_seqs, 14, 2, 64, 16, spec.num_blocks, spec.max_blocks, torch.bfloat16,
                         variant)
    ws = torch.zeros(plan["workspace_bytes"], dtype=torch.uint8, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.empty_like(q)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    st = _native.lib().mvb_test_decode_wait_timeout(
        q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), bt.stride(0),
        bt.shape[1], kvl.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1), spec.num_seqs, 14, 2, 64, 16,
        spec.num_blocks, 0.125, _native.DTYPE_BF16, ws.data_ptr(), ws.numel(), err.data_ptr(),
        torch.cuda.current_stream(DEV).cuda_stream, 7, 2, 4096,
        _native.DECODE_STREAM if variant == "stream" else _native.DECODE_SCHED)
    assert st == _native.OK, _native.status_string(st)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 30.0  # bounded: the held stage gives up after 4096 try-waits
    assert int(err.item()) & _native.DEV_TIMEOUT
    # the host mapping of the bit
    from mini_vllm_b200.attention import paged_attention_b200 as P

    with pytest.raises(RuntimeError, match="timed out"):
        P._raise_flags(int(err.item()), None)
    # the context is still usable: a normal decode is correct
    res = M.paged_decode_attention(q, kc, vc, bt, kvl, 16, variant=variant)
    ref, s2 = oracle.decode(torch_to_np(q, "bf16"), torch_to_np(kc, "bf16"), torch_to_np(vc, "bf16"),
                            spec.block_tables, spec.context_lens, 16, "bf16")
    assert (s2 == 0).all()
    g = res.float().cpu().numpy()
    assert (np.abs(g - ref) <= 2e-3 + 1e-2 * np.abs(ref)).all()
    # the failed call's own workspace serves the next decode: the arrival
    # counters of cut units ended at zero (the timed-out warp still counted its
    # pieces in), so every cut unit is merged again
    err.zero_()
    out2 = torch.full_like(q, 9.0)
    st = _native.lib().mvb_paged_decode(
        q.data_ptr(), q.stride(0), q.stride(1), kc.data_ptr(), vc.data_ptr(), bt.data_ptr(), bt.stride(0),
        bt.shape[1], kvl.data_ptr(), out2.data_ptr(), out2.stride(0), out2.stride(1), spec.num_seqs, 14, 2, 64, 16,
        spec.num_blocks, 0.125, _native.DTYPE_BF16,
        _native.DECODE_STREAM if variant == "stream" else _native.DECODE_SCHED, 0, ws.data_ptr(), ws.numel(),
        err.data_ptr(), torch.cuda.current_stream(DEV).cuda_stream)
    assert st == _native.OK, _native.status_string(st)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    g2 = out2.float().cpu().numpy()
    assert (np.abs(g2 - ref) <= 2e-3 + 1e-2 * np.abs(ref)).all()


def test_hook_rejects_bad_arguments():
    z = 0
    st = _native.lib().mvb_test_decode_wait_timeout(
        None, z, z, None, None, None, z, z, None, None, z, z, 1, 14, 2, 64, 16, 8, 0.125, _native.DTYPE_BF16,
        None, z, None, None, -1, 0, 4096, _native.DECODE_STREAM)
    assert st == _native.ERR_INVALID_ARG
    st = _native.lib().mvb_test_decode_wait_timeout(
        None, z, z, None, None, None, z, z, None, None, z, z, 1, 14, 2, 64, 16, 8, 0.125, _native.DTYPE_BF16,
        None, z, None, None, 0, 0, 4096, _native.DECODE_MMA)
    assert st == _native.ERR_VARIANT
