"""Fused RoPE + KV write (mvb_rope_kv_cache_write) against the reference (GPU).

Bit-exact: the rotated query, the rotated keys and the whole pool after the
write must equal the reference's RotaryEmbedding + write_to_paged_cache
(golden vectors) and the oracle's restatement of them (rope_numpy +
cache_write) on config-2 decode steps and prefill chunks, for every dtype, on
views of a fused QKV output, in place, and on the unaligned (scalar) path.
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


def test_golden_rope_writes_bit_exact(golden):
    cases, arrays = golden
    ran = 0
    for c in [c for c in cases if c["kind"] == "rope"]:
        dt = c["dtype"]
        x = MG.rope_inputs(c)
        cos, sin = M.rope_tables(c["head_dim"], c["theta"], c["max_seq"], TDT[dt])  # CPU: the reference's tables
        kc, vc = np_to_torch(x["kc0"], dt, DEV), np_to_torch(x["vc0"], dt, DEV)
        q_rot, k_rot = M.rope_cache_write(
            np_to_torch(x["q"], dt, DEV), np_to_torch(x["k"], dt, DEV), np_to_torch(x["v"], dt, DEV),
            torch.from_numpy(x["positions"]).to(DEV), cos.to(DEV), sin.to(DEV), kc, vc,
            torch.from_numpy(x["slots"]).to(DEV), c["block_size"], return_key=True)
        assert np.array_equal(torch_to_np(q_rot, dt), arrays[f"{c['name']}/q_rot"]), c["name"]
        assert np.array_equal(torch_to_np(k_rot, dt), arrays[f"{c['name']}/k_rot"]), c["name"]
        assert MG.sha(torch_to_np(kc, dt), torch_to_np(vc, dt)) == c["result_sha256"], c["name"]
        ran += 1
    assert ran >= 5


def _oracle_step(q, k, v, pos, cos, sin, kc, vc, slots, bs, dt):
    """rope(q), rope(k), then the sequential write — on the host."""
    cos_np, sin_np = torch_to_np(cos, dt), torch_to_np(sin, dt)
    p = pos.cpu().numpy()
    q_rot = oracle.rope_numpy(torch_to_np(q, dt), p, cos_np, sin_np, dt)
    k_rot = oracle.rope_numpy(torch_to_np(k, dt), p, cos_np, sin_np, dt)
    kc_np, vc_np = torch_to_np(kc, dt), torch_to_np(vc, dt)
    oracle.cache_write(k_rot, torch_to_np(v, dt), kc_np, vc_np, slots.cpu().numpy(), bs, dt)
    return q_rot, k_rot, kc_np, vc_np


def _fused_qkv(t, h, kh, d, dtype, seed):
    """The QKV projection's output [T, (H + 2 KH) * D] and its q / k / v views."""
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(t, (h + 2 * kh) * d, generator=g).to(dtype).to(DEV)
    q = qkv[:, :h * d].view(t, h, d)
    k = qkv[:, h * d:(h + kh) * d].view(t, kh, d)
    v = qkv[:, (h + kh) * d:].view(t, kh, d)
    return qkv, q, k, v


@pytest.mark.parametrize("dt", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("t,h,kh,d,nb", [(256, 14, 2, 64, 600), (4096, 14, 2, 64, 300), (33, 32, 8, 128, 8)])
def test_rope_write_matches_oracle(dt, t, h, kh, d, nb):
    bs = 16
    _, q, k, v = _fused_qkv(t, h, kh, d, TDT[dt], seed=t + d)
    cos, sin = M.rope_tables(d, 1e6, 40960, TDT[dt], device=DEV)  # built on the device, as the runner does
    g = torch.Generator().manual_seed(7)
    pos = torch.randint(0, 40960, (t,), generator=g).to(DEV)
    slots = torch.randperm(nb * bs, generator=g)[:t].to(DEV)
    slots[::17] = -1
    kc = torch.randn(nb, kh, bs, d, generator=g).to(TDT[dt]).to(DEV)
    vc = torch.randn(nb, kh, bs, d, generator=g).to(TDT[dt]).to(DEV)
    ref_q, ref_k, ref_kc, ref_vc = _oracle_step(q, k, v, pos, cos, sin, kc, vc, slots, bs, dt)
    q_rot, k_rot = M.rope_cache_write(q, k, v, pos, cos, sin, kc, vc, slots, bs, return_key=True)
    assert np.array_equal(torch_to_np(q_rot, dt), ref_q)
    assert np.array_equal(torch_to_np(k_rot, dt), ref_k)
    assert np.array_equal(torch_to_np(kc, dt), ref_kc) and np.array_equal(torch_to_np(vc, dt), ref_vc)


def test_rope_write_in_place_and_unaligned_path():
    """query_out = query (in place), and rows whose strides are not 16-byte
    multiples (the one-element path): same bits as the oracle."""
    t, h, kh, d, bs, nb = 40, 4, 2, 64, 16, 8
    g = torch.Generator().manual_seed(11)
    buf = torch.randn(t, h + 2 * kh, d + 1, generator=g).to(torch.bfloat16).to(DEV)  # row stride d+1
    q, k, v = buf[:, :h, :d], buf[:, h:h + kh, :d], buf[:, h + kh:, :d]
    cos, sin = M.rope_tables(d, 1e4, 256, torch.bfloat16, device=DEV)
    pos = torch.randint(0, 256, (t,), generator=g).to(DEV)
    slots = torch.randperm(nb * bs, generator=g)[:t].to(DEV)
    kc = torch.zeros(nb, kh, bs, d, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    ref_q, ref_k, ref_kc, ref_vc = _oracle_step(q, k, v, pos, cos, sin, kc, vc, slots, bs, "bf16")
    q_rot, _ = M.rope_cache_write(q, k, v, pos, cos, sin, kc, vc, slots, bs)
    assert np.array_equal(torch_to_np(q_rot, "bf16"), ref_q)
    assert np.array_equal(torch_to_np(kc, "bf16"), ref_kc) and np.array_equal(torch_to_np(vc, "bf16"), ref_vc)
    # in place on a contiguous query
    qc = q.contiguous()
    out, _ = M.rope_cache_write(qc, k, v, pos, cos, sin, kc, vc, slots, bs, query_out=qc, check_duplicates=False)
    assert out.data_ptr() == qc.data_ptr()
    assert np.array_equal(torch_to_np(qc, "bf16"), ref_q)


def test_rope_write_errors():
    t, h, kh, d, bs, nb = 4, 2, 1, 64, 16, 2
    q = torch.randn(t, h, d, device=DEV).to(torch.bfloat16)
    k = torch.randn(t, kh, d, device=DEV).to(torch.bfloat16)
    cos, sin = M.rope_tables(d, 1e4, 64, torch.bfloat16, device=DEV)
    kc = torch.zeros(nb, kh, bs, d, dtype=torch.bfloat16, device=DEV)
    vc = torch.zeros_like(kc)
    ok_pos = torch.tensor([0, 1, 2, 63], device=DEV)
    with pytest.raises(IndexError, match="rope position"):
        M.rope_cache_write(q, k, k, torch.tensor([0, 1, 64, 2], device=DEV), cos, sin, kc, vc,
                           torch.arange(t, device=DEV), bs)
    with pytest.raises(IndexError, match="out of range"):
        M.rope_cache_write(q, k, k, ok_pos, cos, sin, kc, vc, torch.tensor([0, 1, 2, 99], device=DEV), bs)
    with pytest.raises(AssertionError, match="Duplicate"):
        M.rope_cache_write(q, k, k, ok_pos, cos, sin, kc, vc, torch.tensor([0, 5, 5, 7], device=DEV), bs)
    with pytest.raises(M.ArgumentError, match="one dtype"):
        M.rope_cache_write(q, k, k, ok_pos, cos.float(), sin.float(), kc, vc, torch.arange(t, device=DEV), bs)
    # the error word is clear afterwards: a good call passes
    M.rope_cache_write(q, k, k, ok_pos, cos, sin, kc, vc, torch.arange(t, device=DEV), bs)
