"""Stream-ordered staging helpers (mini_vllm_b200.staging) on the GPU.

A serving loop's copies: H2D of inputs on a side stream, the compute stream
waits for them, computes, and the D2H of the result on the side stream waits
for the compute.  The helpers must order the work exactly as torch's
copy_ / wait_event / record do, step after step with reused buffers.
"""

from __future__ import annotations

import pytest
import torch

import mini_vllm_b200 as M

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_staged_h2d_compute_d2h_in_order():
    n = 1 << 20
    side = torch.cuda.Stream(DEV)
    compute = torch.cuda.current_stream(DEV)
    host_in = [torch.empty(n, dtype=torch.float32).pin_memory() for _ in range(2)]
    host_out = [torch.empty(n, dtype=torch.float32).pin_memory() for _ in range(2)]
    dev_in = [torch.empty(n, dtype=torch.float32, device=DEV) for _ in range(2)]
    dev_out = [torch.empty(n, dtype=torch.float32, device=DEV) for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    done = [torch.cuda.Event() for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    results = []
    for step in range(6):
        b = step & 1
        if step >= 2:  # the host buffers of this slot are free once their D2H is done
            copied[b].synchronize()
            results.append((step - 2, host_out[b].clone()))
        host_in[b].fill_(float(step))
        # H2D waits for the last compute that read this slot (never recorded at first: skipped)
        M.staging.stream_copy(dev_in[b], host_in[b], side, wait=done[b], record=in_ready[b])
        M.staging.wait_events(compute, in_ready[b], copied[b])
        torch.mul(dev_in[b], 3.0, out=dev_out[b])
        M.staging.record(done[b], compute)
        M.staging.stream_copy(host_out[b], dev_out[b], side, wait=done[b], record=copied[b])
    torch.cuda.synchronize()
    for b in range(2):
        results.append((4 + b, host_out[b].clone()))
    assert sorted(s for s, _ in results) == list(range(6))
    for step, out in results:
        assert torch.equal(out, torch.full((n,), 3.0 * step))


def test_staging_errors():
    side = torch.cuda.Stream(DEV)
    with pytest.raises(ValueError, match="exactly one"):
        M.staging.stream_copy(torch.zeros(4, device=DEV), torch.zeros(4, device=DEV), side)
    with pytest.raises(ValueError, match="size"):
        M.staging.stream_copy(torch.zeros(4, device=DEV), torch.zeros(8).pin_memory(), side)


def test_staging_rejects_a_stream_of_another_device():
    """The device tensor and the stream must be on the same GPU (checked
    before any CUDA call: the stream here only claims another device)."""
    import types

    other = types.SimpleNamespace(device=torch.device("cuda", DEV.index + 1), cuda_stream=0)
    with pytest.raises(ValueError, match="stream belongs to"):
        M.staging.stream_copy(torch.zeros(4, device=DEV), torch.zeros(4).pin_memory(), other)


def test_copy_plan_repeats_the_checked_copy():
    """A CopyPlan, checked once, copies its fixed tensors on every run: host
    to device, a kernel in between, device to host, ordered by its events."""
    dev = torch.device("cuda", 0)
    side = torch.cuda.Stream(dev)
    host_in = torch.empty(1 << 16, dtype=torch.float32).pin_memory()
    host_out = torch.empty(1 << 16, dtype=torch.float32).pin_memory()
    dbuf = torch.empty(1 << 16, dtype=torch.float32, device=dev)
    dout = torch.empty_like(dbuf)
    ready, done, copied = torch.cuda.Event(), torch.cuda.Event(), torch.cuda.Event()
    h2d = M.staging.CopyPlan(dbuf, host_in, side, wait=done, record=ready)
    d2h = M.staging.CopyPlan(host_out, dout, side, wait=done, record=copied)
    compute = torch.cuda.current_stream(dev)
    for step in range(5):
        host_in.fill_(float(step))
        h2d.run()
        M.staging.wait_events(compute, ready)
        torch.mul(dbuf, 2.0, out=dout)
        M.staging.record(done, compute)
        d2h.run()
        copied.synchronize()
        assert (host_out == 2.0 * step).all()
    with pytest.raises(ValueError, match="exactly one"):
        M.staging.CopyPlan(dbuf, dout, side)
