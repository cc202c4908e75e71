"""The paged prefill kernel (mvb_paged_prefill) against a float32 torch
reference of the reference backend's prefill math (GPU).

AttentionBackendGPU.prefill_attention (mini_vllm/attention/paged_attention_gpu.py:
577-661) gathers each sequence's cached prefix, appends the chunk's K/V,
repeats the KV heads for GQA and runs SDPA with the offset causal mask
(key position <= cached + query index).  The kernel reads the prefix in place
from the pool.  Cases: chunks from 1 to 300 tokens with prefixes from 0 to
1000 tokens, GQA 1 / 4 / 7 / 16 (two CTA head groups), head_dim 64 and 128,
block sizes 8 to 64, bf16 and f16, the chunk read from key / value or from the
cache, 300 chunks in one launch, and the error paths.  Tolerance: the decode
parity bound 2e-3 + 1e-2 |ref|.
"""

from __future__ import annotations

import pytest
import torch

import mini_vllm_b200 as M
from mini_vllm_b200 import _native

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _ref(q, k, v, cached, reps):
    """float32 SDPA with the offset causal mask, GQA by repetition."""
    qf, kf, vf = q.float(), k.float().repeat_interleave(reps, 1), v.float().repeat_interleave(reps, 1)
    kv_len, q_len = kf.shape[0], qf.shape[0]
    mask = torch.arange(kv_len, device=q.device)[None, :] <= torch.arange(cached, cached + q_len,
                                                                          device=q.device)[:, None]
    o = torch.nn.functional.scaled_dot_product_attention(
        qf.permute(1, 0, 2)[None], kf.permute(1, 0, 2)[None], vf.permute(1, 0, 2)[None], attn_mask=mask,
        scale=q.shape[-1] ** -0.5)
    return o[0].permute(1, 0, 2)


def _close(a, b, msg=""):
    err = (a.float() - b).abs()
    assert torch.isfinite(a.float()).all(), msg
    assert (err <= 2e-3 + 1e-2 * b.abs()).all(), f"{msg}: max abs err {err.max().item():.3e}"


def _case(seqs, h, kh, d, bs, dtype, seed=0, garbage_chunk=False):
    """A pool holding every sequence's context (cached + chunk) at shuffled
    blocks; with garbage_chunk the chunk's positions in the pool hold other
    values (so a read of the chunk from the cache would be wrong)."""
    g = torch.Generator().manual_seed(seed)
    need = [(c + n + bs - 1) // bs for c, n in seqs]
    nb = sum(need) + 3
    perm = torch.randperm(nb, generator=g)
    table = torch.full((len(seqs) + 2, max(need) + 1), -1, dtype=torch.int64)
    rows = torch.randperm(len(seqs) + 2, generator=g)[:len(seqs)]  # chunks use scattered table rows
    kc = torch.randn(nb, kh, bs, d, generator=g).to(dtype).to(DEV)
    vc = torch.randn(nb, kh, bs, d, generator=g).to(dtype).to(DEV)
    pos = 0
    ks, vs, qs = [], [], []
    for i, (c, n) in enumerate(seqs):
        table[rows[i], :need[i]] = perm[pos:pos + need[i]]
        pos += need[i]
        k = torch.randn(c + n, kh, d, generator=g).to(dtype).to(DEV)
        v = torch.randn(c + n, kh, d, generator=g).to(dtype).to(DEV)
        p = torch.arange(c + n)
        slots = (table[rows[i]][p // bs] * bs + p % bs).to(DEV)
        if garbage_chunk:
            M.paged_cache_write(k[:c], v[:c], kc, vc, slots[:c], bs)
            M.paged_cache_write(-k[c:], v[c:] * 3, kc, vc, slots[c:], bs)
        else:
            M.paged_cache_write(k, v, kc, vc, slots, bs)
        ks.append(k)
        vs.append(v)
        qs.append(torch.randn(n, h, d, generator=g).to(dtype).to(DEV))
    return kc, vc, table.to(DEV), rows, ks, vs, qs


@pytest.mark.parametrize("h,kh,d,bs", [(14, 2, 64, 16), (32, 8, 128, 16), (32, 2, 64, 32), (8, 8, 64, 8),
                                       (14, 2, 128, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("with_chunk", [True, False])
def test_prefill_matches_the_reference_math(h, kh, d, bs, dtype, with_chunk):
    seqs = [(0, 1), (0, 17), (5, 16), (100, 33), (1000, 300), (37, 5), (16, 15)]
    kc, vc, table, rows, ks, vs, qs = _case(seqs, h, kh, d, bs, dtype, seed=h + d + bs,
                                            garbage_chunk=with_chunk)
    q = torch.cat(qs)
    chunk_k = torch.cat([k[c:] for k, (c, _) in zip(ks, seqs)]) if with_chunk else None
    chunk_v = torch.cat([v[c:] for v, (c, _) in zip(vs, seqs)]) if with_chunk else None
    out = M.paged_prefill_attention(q, kc, vc, table, rows, [c for c, _ in seqs], [n for _, n in seqs], bs,
                                    key=chunk_k, value=chunk_v)
    assert out.shape == q.shape and out.dtype == dtype
    off = 0
    for i, (c, n) in enumerate(seqs):
        _close(out[off:off + n], _ref(qs[i], ks[i], vs[i], c, h // kh), f"chunk {i} ({c}+{n})")
        off += n


def test_many_chunks_in_one_launch_and_device_metadata():
    """300 chunks (the CTA's tile prefix spans many sequences); metadata as
    int64 device tensors, the form that needs no host synchronisation."""
    g = torch.Generator().manual_seed(3)
    seqs = [(int(c), int(n)) for c, n in zip(torch.randint(0, 200, (300,), generator=g),
                                              torch.randint(1, 40, (300,), generator=g))]
    kc, vc, table, rows, ks, vs, qs = _case(seqs, 14, 2, 64, 16, torch.bfloat16, seed=4)
    q = torch.cat(qs)
    cached = torch.tensor([c for c, _ in seqs], device=DEV)
    qlen = torch.tensor([n for _, n in seqs], device=DEV)
    out = M.paged_prefill_attention(q, kc, vc, table, rows.to(DEV), cached, qlen, 16, strict=False)
    M.check_device_errors()
    off = 0
    for i, (c, n) in enumerate(seqs):
        _close(out[off:off + n], _ref(qs[i], ks[i], vs[i], c, 7), f"chunk {i}")
        off += n


def test_backend_prefill_uses_the_kernel_for_every_group():
    """The backend's prefill_attention: every prefill group of the step in one
    launch, with the chunk's K / V given (the Triton backend's form)."""
    seqs = [(0, 12), (8, 2), (300, 64)]
    kc, vc, table, rows, ks, vs, qs = _case(seqs, 14, 2, 64, 16, torch.float16, seed=9)
    backend = M.AttentionBackendB200(M.ModelConfig(num_heads=14, num_kv_heads=2, head_dim=64))
    pool = M.KVCachePool([kc], [vc], kc.shape[0], 16, 1, 2, 64, DEV, torch.float16)
    groups = [M.AttentionGroup(seq_indices=[int(rows[i])], attention_type="prefill_gpu",
                               cached_len_before=torch.tensor([c], device=DEV), query_len=torch.tensor([n], device=DEV),
                               kv_len_after=torch.tensor([c + n], device=DEV)) for i, (c, n) in enumerate(seqs)]
    meta = M.AttentionMetadata(groups=groups, prefill_block_tables=table, block_size=16, num_kv_heads=2, head_dim=64)
    q = torch.cat(qs)
    nk = torch.cat([k[c:] for k, (c, _) in zip(ks, seqs)])
    nv = torch.cat([v[c:] for v, (c, _) in zip(vs, seqs)])
    out = backend.prefill_attention(0, q, nk, nv, meta, pool)
    off = 0
    for i, (c, n) in enumerate(seqs):
        _close(out[off:off + n], _ref(qs[i], ks[i], vs[i], c, 7), f"group {i}")
        off += n


def test_short_table_gives_zero_rows_and_raises():
    seqs = [(20, 10), (3, 4)]
    kc, vc, table, rows, ks, vs, qs = _case(seqs, 14, 2, 64, 16, torch.bfloat16, seed=5)
    q = torch.cat(qs)
    # the first chunk claims 40 cached tokens: its end (50) needs 4 blocks, the table has 3 columns
    narrow = table[:, :3].contiguous()
    with pytest.raises(IndexError):
        M.paged_prefill_attention(q, kc, vc, narrow, rows, [40, 3], [10, 4], 16)
    out = M.paged_prefill_attention(q, kc, vc, narrow, rows, [40, 3], [10, 4], 16, strict=False)
    with pytest.raises(IndexError, match="block_table length insufficient"):
        M.check_device_errors()
    assert (out[:10] == 0).all()
    _close(out[10:], _ref(qs[1], ks[1], vs[1], 3, 7))


def test_more_chunk_tokens_than_query_rows_is_refused():
    """query_len summing past the query's rows: the kernel refuses (flag) and
    writes nothing — it never reads or writes past the tensors."""
    seqs = [(0, 8)]
    kc, vc, table, rows, ks, vs, qs = _case(seqs, 14, 2, 64, 16, torch.bfloat16, seed=6)
    q = qs[0]
    out = torch.full_like(q, 7.0)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    r64 = rows.to(DEV)
    c64 = torch.tensor([0], device=DEV)
    n64 = torch.tensor([40], device=DEV)
    st = _native.lib().mvb_paged_prefill(
        q.data_ptr(), q.stride(0), q.stride(1), None, 0, 0, None, 0, 0, kc.data_ptr(), vc.data_ptr(),
        table.data_ptr(), table.shape[0], table.stride(0), table.shape[1], r64.data_ptr(), c64.data_ptr(),
        n64.data_ptr(), 1, q.shape[0], out.data_ptr(), out.stride(0), out.stride(1), 14, 2, 64, 16, kc.shape[0],
        0.125, _native.DTYPE_BF16, err.data_ptr(), torch.cuda.current_stream(DEV).cuda_stream)
    assert st == _native.OK
    torch.cuda.synchronize()
    assert int(err.item()) & _native.DEV_BLOCK_ID
    assert (out == 7.0).all()


def test_host_checks():
    lib = _native.lib()
    z = 0
    call = lambda dt=_native.DTYPE_BF16, d=64, bs=16, nc=1, k=None, v=None: lib.mvb_paged_prefill(
        16, z, z, k, z, z, v, z, z, 16, 16, 16, 1, 1, 1, 16, 16, 16, nc, 8, 16, z, z, 14, 2, d, bs, 4, 0.125, dt, 16,
        None)
    assert call(dt=_native.DTYPE_F32) == _native.ERR_DTYPE
    assert call(d=80) == _native.ERR_HEAD_DIM
    assert call(bs=12) == _native.ERR_BLOCK_SIZE
    assert call(nc=5000) == _native.ERR_INVALID_ARG
    assert call(k=16) == _native.ERR_INVALID_ARG  # key without value
    assert call(nc=0) == _native.OK
