"""Paged decode kernels vs the oracle / reference golden vectors (GPU).

Tolerance (the north star's, in allclose form): for bf16 / f16,
    |gpu - ref| <= 2e-3 + 1e-2 * |ref|
element-wise, where ref is the reference computed in fp32 on the same
(upcast) inputs and gpu is the kernel's output in the query dtype, widened.
fp32 runs use 1e-4 + 1e-4 * |ref|.

Ports the reference's TestDecodeAttention / TestGQA
(test_paged_attention_gpu.py:215-825) and adds BASELINE-size configs 2, 3, 4,
both kernel variants, forced split-K and the error contract.
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
TDT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def tol(dtype: str):
    return (1e-4, 1e-4) if dtype == "f32" else (2e-3, 1e-2)


def assert_close(gpu: torch.Tensor, ref: np.ndarray, dtype: str, msg: str = ""):
    atol, rtol = tol(dtype)
    g = gpu.float().cpu().numpy()
    assert np.isfinite(g).all(), f"non-finite output {msg}"
    err = np.abs(g - ref)
    bound = atol + rtol * np.abs(ref)
    if msg.startswith("config"):
        # the observed margins, for the record (pytest -s prints them): max abs,
        # and max rel over outputs with |ref| >= 1e-2 (below, bf16 rounding of the
        # output alone exceeds 1 % relative)
        big = np.abs(ref) >= 1e-2
        rel = (err[big] / np.abs(ref[big])).max() if big.any() else 0.0
        print(f"PARITY {msg}: max_abs={err.max():.3e} max_rel(|ref|>=1e-2)={rel:.3e} "
              f"max_err/bound={(err / bound).max():.3f}")
    worst = np.unravel_index(np.argmax(err - bound), err.shape)
    assert (err <= bound).all(), (
        f"{msg}: max excess at {worst}: gpu={g[worst]} ref={ref[worst]} "
        f"(max abs err {err.max():.3e})")


def variants_for(dtype: str, block_size: int, head_dim: int):
    v = ["auto", "fma"]
    if dtype != "f32" and block_size % 16 == 0 and head_dim in (64, 128):
        v += ["mma", "stream", "sched"]
    return v


def run(x, dtype, variant="auto", partition_tokens=None, **kw):
    q = np_to_torch(x["q"], dtype, DEV)
    kc, vc = np_to_torch(x["kc"], dtype, DEV), np_to_torch(x["vc"], dtype, DEV)
    bt = torch.from_numpy(np.asarray(x["tables"], np.int64)).to(DEV)
    kvl = torch.from_numpy(np.asarray(x["ctx"], np.int32)).to(DEV)
    return M.paged_decode_attention(q, kc, vc, bt, kvl, x["block_size"], variant=variant,
                                    partition_tokens=partition_tokens, **kw)


@pytest.mark.parametrize("kind", ["decode", "decode_spec"])
def test_golden_decodes_all_variants(golden, kind):
    cases, arrays = golden
    ran = 0
    for c in [c for c in cases if c["kind"] == kind]:
        x = MG.decode_inputs(c)
        d = x["q"].shape[2]
        if d not in (64, 128):
            with pytest.raises(AssertionError, match="head_dim"):
                run(x, c["dtype"])
            continue
        ref = arrays[f"{c['name']}/out"]
        for v in variants_for(c["dtype"], x["block_size"], d):
            out = run(x, c["dtype"], v)
            assert out.dtype == TDT[c["dtype"]]
            assert_close(out, ref, c["dtype"], f"{c['name']} [{v}]")
            ran += 1
    assert ran > 0


@pytest.mark.parametrize("variant,partition_tokens", [
    ("sched", None), ("stream", None), ("mma", None), ("mma", 16), ("mma", 48), ("mma", 512), ("mma", 1024),
    ("fma", None), ("fma", 512),
])
def test_config2_full_size_vs_oracle(variant, partition_tokens):
    """BASELINE config 2 (256 seqs, ctx U[128,2048], 14/2/64, bf16) at full size."""
    spec = W.make_spec(2, seed=21)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                   t["kv_len"], spec.block_size, variant=variant,
                                   partition_tokens=partition_tokens)
    ref, st = oracle.decode(torch_to_np(t["query"], "bf16"), torch_to_np(t["key_caches"][0], "bf16"),
                            torch_to_np(t["value_caches"][0], "bf16"), spec.block_tables,
                            spec.context_lens, spec.block_size, "bf16")
    assert (st == 0).all()
    assert_close(out, ref, "bf16", f"config2 {variant} pt={partition_tokens}")


def test_config3_long_context_split_k_vs_oracle():
    """32 x 32768 tokens — flash-decoding 512-token partitions
    plus the reduction kernel, and the stream kernel."""
    spec = W.make_spec(3, seed=0)
    plan = M.decode_plan(spec.num_seqs, 14, 2, 64, 16, spec.num_blocks, spec.max_blocks, torch.bfloat16,
                         variant="mma")
    assert plan["num_partitions"] == 64 and plan["partition_tokens"] == 512
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    ref, st = oracle.decode(torch_to_np(t["query"], "bf16"), torch_to_np(t["key_caches"][0], "bf16"),
                            torch_to_np(t["value_caches"][0], "bf16"), spec.block_tables,
                            spec.context_lens, spec.block_size, "bf16")
    assert (st == 0).all()
    for v in ("mma", "stream", "sched"):
        out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0],
                                       t["block_tables"], t["kv_len"], spec.block_size, variant=v)
        assert_close(out, ref, "bf16", f"config3 {v}")


@pytest.mark.parametrize("variant", ["sched", "stream", "mma", "fma"])
def test_config4_gqa4_d128_vs_oracle(variant):
    """BASELINE config 4 shape (32/8/128, lognormal ctx), a 96-sequence shard."""
    spec = W.make_spec(4, seed=2, num_seqs=96)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                   t["kv_len"], spec.block_size, variant=variant)
    ref, st = oracle.decode(torch_to_np(t["query"], "bf16"), torch_to_np(t["key_caches"][0], "bf16"),
                            torch_to_np(t["value_caches"][0], "bf16"), spec.block_tables,
                            spec.context_lens, spec.block_size, "bf16")
    assert (st == 0).all()
    assert_close(out, ref, "bf16", f"config4 {variant}")


@pytest.mark.parametrize("dtype", ["f16", "f32"])
def test_config1_vs_oracle_other_dtypes(dtype):
    spec = W.make_spec(1, seed=3)
    t = W.torch_tensors(spec, TDT[dtype], DEV)
    out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                   t["kv_len"], spec.block_size)
    ref, _ = oracle.decode(torch_to_np(t["query"], dtype), torch_to_np(t["key_caches"][0], dtype),
                           torch_to_np(t["value_caches"][0], dtype), spec.block_tables, spec.context_lens,
                           spec.block_size, dtype)
    assert_close(out, ref, dtype, f"config1 {dtype}")


@pytest.mark.parametrize("block_size", [1, 2, 8, 32, 64, 128])
def test_block_sizes(block_size):
    ctx = np.array([1, 15, 16, 17, 200, 513], dtype=np.int64)
    spec = W.build_spec("bs", ctx, 8, 2, 64, block_size, seed=block_size)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    ref, _ = oracle.decode(torch_to_np(t["query"], "bf16"), torch_to_np(t["key_caches"][0], "bf16"),
                           torch_to_np(t["value_caches"][0], "bf16"), spec.block_tables, spec.context_lens,
                           block_size, "bf16")
    for v in variants_for("bf16", block_size, 64):
        out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0],
                                       t["block_tables"], t["kv_len"], block_size, variant=v)
        assert_close(out, ref, "bf16", f"bs={block_size} {v}")


@pytest.mark.parametrize("heads", [(2, 2), (4, 2), (16, 2), (32, 2), (40, 8), (6, 1)])
def test_gqa_group_sizes(heads):
    """G = 1..20 query heads per KV head (head groups split over CTAs above 16 / 8)."""
    h, kh = heads
    ctx = np.array([5, 64, 333], dtype=np.int64)
    spec = W.build_spec("gqa", ctx, h, kh, 128 if h == 40 else 64, 16, seed=h)
    t = W.torch_tensors(spec, torch.float16, DEV)
    ref, _ = oracle.decode(torch_to_np(t["query"], "f16"), torch_to_np(t["key_caches"][0], "f16"),
                           torch_to_np(t["value_caches"][0], "f16"), spec.block_tables, spec.context_lens,
                           16, "f16")
    for v in ("sched", "stream", "mma", "fma"):
        out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0],
                                       t["block_tables"], t["kv_len"], 16, variant=v)
        assert_close(out, ref, "f16", f"G={h // kh} {v}")


def test_strided_query_and_out_param():
    """Query as a non-contiguous view (decode slice of a fused QKV output)."""
    spec = W.build_spec("q", np.array([40, 77, 128, 3], np.int64), 14, 2, 64, 16, seed=9)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    T = 10  # 6 prefill tokens + 4 decode tokens
    qkv = torch.randn(T, 18, 64, device=DEV, dtype=torch.bfloat16)
    q = qkv[6:, :14]
    assert not q.is_contiguous()
    out = torch.full((4, 14, 64), float("nan"), device=DEV, dtype=torch.bfloat16)
    res = M.paged_decode_attention(q, t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                   t["kv_len"], 16, out=out)
    assert res.data_ptr() == out.data_ptr()
    ref, _ = oracle.decode(torch_to_np(q.contiguous(), "bf16"), torch_to_np(t["key_caches"][0], "bf16"),
                           torch_to_np(t["value_caches"][0], "bf16"), spec.block_tables, spec.context_lens,
                           16, "bf16")
    assert_close(out, ref, "bf16", "strided query")


def test_custom_scale():
    spec = W.build_spec("s", np.array([50, 300], np.int64), 8, 2, 64, 16, seed=4)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"],
                                   t["kv_len"], 16, scale=0.3)
    ref, _ = oracle.decode(torch_to_np(t["query"], "bf16"), torch_to_np(t["key_caches"][0], "bf16"),
                           torch_to_np(t["value_caches"][0], "bf16"), spec.block_tables, spec.context_lens,
                           16, "bf16", scale=0.3)
    assert_close(out, ref, "bf16", "scale 0.3")


def test_nan_garbage_past_context_is_never_used():
    """Pool memory past kv_len is torch.empty garbage; fill it with NaN/Inf."""
    ctx = np.array([1, 17, 30], np.int64)
    spec = W.build_spec("nan", ctx, 14, 2, 64, 16, seed=5)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    kc, vc = t["key_caches"][0], t["value_caches"][0]
    for s, n in enumerate(ctx.tolist()):
        last = int(spec.block_tables[s][(n - 1) // 16])
        kc[last, :, (n % 16 or 16):] = float("nan")
        vc[last, :, (n % 16 or 16):] = float("inf")
    for v in ("sched", "stream", "mma", "fma"):
        out = M.paged_decode_attention(t["query"], kc, vc, t["block_tables"], t["kv_len"], 16, variant=v)
        assert torch.isfinite(out.float()).all(), v
    ref, _ = oracle.decode(torch_to_np(t["query"], "bf16"), torch_to_np(kc, "bf16"), torch_to_np(vc, "bf16"),
                           spec.block_tables, spec.context_lens, 16, "bf16")
    assert_close(out, ref, "bf16", "nan garbage")


@pytest.mark.parametrize("variant", ["sched", "stream", "mma", "fma"])
def test_deterministic_bits(variant):
    spec = W.make_spec(2, seed=8, num_seqs=64)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    args = (t["query"], t["key_caches"][0], t["value_caches"][0], t["block_tables"], t["kv_len"], 16)
    a = M.paged_decode_attention(*args, variant=variant)
    for _ in range(3):
        assert torch.equal(a, M.paged_decode_attention(*args, variant=variant))


@pytest.mark.parametrize("num_seqs", [1, 2, 5, 37, 300, 1500, 4000, 64])
def test_stream_kernel_batch_sizes(num_seqs):
    """Few sequences (fewer tiles than warps: empty warp ranges), one sequence
    split across many warps, and large batches (many units per warp)."""
    ctx = W.context_lengths(2, seed=num_seqs, num_seqs=num_seqs)
    if num_seqs <= 2:
        ctx[:] = [3000, 1][:num_seqs]
    spec = W.build_spec("b", ctx, 14, 2, 64, 16, seed=num_seqs)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    ref, _ = oracle.decode(torch_to_np(t["query"], "bf16"), torch_to_np(t["key_caches"][0], "bf16"),
                           torch_to_np(t["value_caches"][0], "bf16"), spec.block_tables, spec.context_lens,
                           16, "bf16")
    for _ in range(2):  # the second call reuses the counters the first left at zero
        out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0],
                                       t["block_tables"], t["kv_len"], 16, variant="stream")
        assert_close(out, ref, "bf16", f"stream n={num_seqs}")


@pytest.mark.parametrize("head_dim,heads,kv_heads", [(64, 14, 2), (128, 32, 8)])
def test_stream_long_units_many_contributors(head_dim, heads, kv_heads):
    """More tiles than warps, and units thousands of tiles long: each is cut
    into hundreds of warp ranges, so the fixup merges more contributors than a
    warp has lanes, in several groups of 32."""
    ctx = np.array([40000, 5, 30001, 17], np.int64)
    spec = W.build_spec("long", ctx, heads, kv_heads, head_dim, 16, seed=41)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    ref, _ = oracle.decode(torch_to_np(t["query"], "bf16"), torch_to_np(t["key_caches"][0], "bf16"),
                           torch_to_np(t["value_caches"][0], "bf16"), spec.block_tables, spec.context_lens,
                           16, "bf16")
    for _ in range(2):
        out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0],
                                       t["block_tables"], t["kv_len"], 16, variant="stream")
        assert_close(out, ref, "bf16", f"stream long D={head_dim}")


# --------------------------------------------------------------------------- errors
def _small():
    kc = torch.randn(8, 2, 16, 64, device=DEV).to(torch.bfloat16)
    q = torch.randn(2, 4, 64, device=DEV).to(torch.bfloat16)
    return q, kc, kc.clone()


@pytest.mark.parametrize("variant", ["sched", "stream", "mma", "fma"])
def test_kv_len_zero_raises_value_error(variant):
    q, kc, vc = _small()
    bt = torch.tensor([[0, -1], [1, 2]], device=DEV)
    kvl = torch.tensor([0, 20], dtype=torch.int32, device=DEV)
    with pytest.raises(ValueError, match="kv_len"):
        M.triton_decode_attention(q, kc, vc, bt, kvl, 16, variant=variant)


@pytest.mark.parametrize("variant", ["sched", "stream", "mma", "fma"])
def test_table_too_short_raises_index_error(variant):
    q, kc, vc = _small()
    bt = torch.tensor([[0], [1]], device=DEV)
    kvl = torch.tensor([10, 20], dtype=torch.int32, device=DEV)
    with pytest.raises(IndexError, match="insufficient"):
        M.paged_decode_attention(q, kc, vc, bt, kvl, 16, variant=variant)


@pytest.mark.parametrize("variant", ["sched", "stream", "mma", "fma"])
@pytest.mark.parametrize("bad", [-1, 8, 1 << 40])
def test_bad_block_id_within_context_raises(variant, bad):
    q, kc, vc = _small()
    bt = torch.tensor([[0, bad], [1, 2]], device=DEV)
    kvl = torch.tensor([20, 20], dtype=torch.int32, device=DEV)
    with pytest.raises(IndexError, match="block_table entry"):
        M.paged_decode_attention(q, kc, vc, bt, kvl, 16, variant=variant)


def test_padding_entries_past_context_are_not_read():
    q, kc, vc = _small()
    bt = torch.tensor([[3, 1 << 40, -7], [1, 2, -1]], device=DEV)  # junk past ctx
    kvl = torch.tensor([16, 20], dtype=torch.int32, device=DEV)
    out = M.paged_decode_attention(q, kc, vc, bt, kvl, 16)
    assert torch.isfinite(out.float()).all()


def test_empty_batch_and_argument_errors():
    q, kc, vc = _small()
    e = q[:0]
    out = M.paged_decode_attention(e, kc, vc, torch.empty(0, 2, dtype=torch.long, device=DEV),
                                   torch.empty(0, dtype=torch.int32, device=DEV), 16)
    assert out.shape == (0, 4, 64)
    bt = torch.tensor([[0, 1], [2, 3]], device=DEV)
    kvl = torch.tensor([3, 3], dtype=torch.int32, device=DEV)
    with pytest.raises(AssertionError, match="power of 2"):
        M.paged_decode_attention(q, kc, vc, bt, kvl, 12)
    with pytest.raises(AssertionError, match="dtype"):
        M.paged_decode_attention(q.half(), kc, vc, bt, kvl, 16)
    with pytest.raises(AssertionError, match="divisible"):
        M.paged_decode_attention(q[:, :3], kc, vc, bt, kvl, 16)


def test_int64_kv_len_and_cpu_metadata_are_accepted():
    q, kc, vc = _small()
    bt = torch.tensor([[0, 1], [2, 3]])
    kvl = torch.tensor([3, 30])
    a = M.paged_decode_attention(q, kc, vc, bt, kvl, 16)
    b = M.paged_decode_attention(q, kc, vc, bt.to(DEV), kvl.to(DEV, torch.int32), 16)
    assert torch.equal(a, b)


def test_stream_and_split_k_calls_interleave():
    """Split-K partials and the stream kernel's arrival counters live in separate
    workspaces: a split call between two stream calls must not disturb them."""
    spec = W.make_spec(2, seed=30, num_seqs=16)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    ref, _ = oracle.decode(torch_to_np(t["query"], "bf16"), torch_to_np(t["key_caches"][0], "bf16"),
                           torch_to_np(t["value_caches"][0], "bf16"), spec.block_tables, spec.context_lens,
                           16, "bf16")
    for v, pt in [("stream", None), ("mma", 256), ("stream", None), ("fma", 128), ("stream", None)]:
        out = M.paged_decode_attention(t["query"], t["key_caches"][0], t["value_caches"][0],
                                       t["block_tables"], t["kv_len"], 16, variant=v, partition_tokens=pt)
        assert_close(out, ref, "bf16", f"{v} pt={pt}")


def test_direct_binding_and_ctypes_route_agree(monkeypatch):
    """The C++ binding (the common case) and the ctypes route (taken when the
    binding declines) launch the same kernels: identical bytes for the write
    and the decode, and the binding is what ran first."""
    from mini_vllm_b200 import _native

    spec = W.make_spec(2, seed=5, num_seqs=64)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    kc_a, vc_a = t["key_caches"][0].clone(), t["value_caches"][0].clone()
    M.paged_cache_write(t["new_key"], t["new_value"], kc_a, vc_a, t["slot_mapping"], 16)
    a = M.paged_decode_attention(t["query"], kc_a, vc_a, t["block_tables"], t["kv_len"], 16)
    assert _native._fast is not None

    class Declines:
        SLOW_PATH = -1000

        @staticmethod
        def kv_write(*args):
            return Declines.SLOW_PATH

        @staticmethod
        def decode(*args):
            return Declines.SLOW_PATH, None

    monkeypatch.setattr(_native, "fast", lambda: Declines)
    kc_b, vc_b = t["key_caches"][0].clone(), t["value_caches"][0].clone()
    M.paged_cache_write(t["new_key"], t["new_value"], kc_b, vc_b, t["slot_mapping"], 16)
    b = M.paged_decode_attention(t["query"], kc_b, vc_b, t["block_tables"], t["kv_len"], 16)
    assert torch.equal(kc_a, kc_b) and torch.equal(vc_a, vc_b)
    assert torch.equal(a, b)


def _write_then_decode_case(seed: int, num_seqs: int):
    """Config-2 shapes whose new tokens dominate attention: K = 4, V = 3 at
    every new slot, so a decode that read the cache before the write landed
    would be far outside tolerance, not just a few ulps off."""
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


@pytest.mark.parametrize("num_seqs", [256, 7])
def test_decode_after_write_overlap_sees_the_write(num_seqs):
    """after_write=True (set-up overlapped with the preceding KV write, no host
    sync in between) gives the oracle's write-then-decode result, bit-identical
    to the ordered launch."""
    spec, t, ref = _write_then_decode_case(31, num_seqs)
    outs = {}
    for flag in (False, True, True):
        kc, vc = t["key_caches"][0].clone(), t["value_caches"][0].clone()
        torch.cuda.synchronize()
        M.paged_cache_write(t["new_key"], t["new_value"], kc, vc, t["slot_mapping"], 16, strict=False)
        o = M.paged_decode_attention(t["query"], kc, vc, t["block_tables"], t["kv_len"], 16, strict=False,
                                     after_write=flag)
        M.check_device_errors()
        assert_close(o, ref, "bf16", f"after_write={flag}")
        if flag in outs:
            assert torch.equal(o, outs[flag])
        outs[flag] = o
    assert torch.equal(outs[False], outs[True])


def test_backend_overlap_after_write_only_for_the_adjacent_decode():
    """The backend passes after_write only to the decode that directly follows
    its own write of the same layer; results match the oracle either way."""
    spec, t, ref = _write_then_decode_case(32, 64)
    backend = M.AttentionBackendB200(M.ModelConfig(num_heads=14, num_kv_heads=2, head_dim=64), strict=False,
                                     overlap_after_write=True)
    kcs = [t["key_caches"][0].clone(), t["key_caches"][0].clone()]
    vcs = [t["value_caches"][0].clone(), t["value_caches"][0].clone()]
    pool = M.KVCachePool(kcs, vcs, spec.num_blocks, 16, 2, 2, 64, torch.device(DEV), torch.bfloat16)
    backend._pool = pool
    group = M.AttentionGroup(seq_indices=list(range(spec.num_seqs)), attention_type="decode_gpu",
                             cached_len_before=None, query_len=None, kv_len_after=t["kv_len"])
    meta = M.AttentionMetadata(groups=[group], decode_block_tables=t["block_tables"], block_size=16,
                               num_kv_heads=2, head_dim=64)
    backend.write_kv_cache(0, t["new_key"], t["new_value"], t["slot_mapping"])
    assert backend._last_write is not None
    a = backend.decode_attention(0, t["query"], meta, pool)
    assert backend._last_write is None
    backend.write_kv_cache(1, t["new_key"], t["new_value"], t["slot_mapping"])
    b = backend.decode_attention(0, t["query"], meta, pool)  # another layer's write: no overlap
    M.check_device_errors()
    assert_close(a, ref, "bf16", "adjacent")
    assert torch.equal(a, b)


def test_backend_decode_into_runner_slice():
    """decode_attention(out=attn_out[num_prefill:]) writes the decode rows in
    place (no allocation, no slice copy) with the same bits as the returning
    form."""
    spec = W.make_spec(2, seed=12, num_seqs=48)
    t = W.torch_tensors(spec, torch.bfloat16, DEV)
    backend = M.AttentionBackendB200(M.ModelConfig(num_heads=14, num_kv_heads=2, head_dim=64))
    pool = M.KVCachePool([t["key_caches"][0]], [t["value_caches"][0]], spec.num_blocks, 16, 1, 2, 64,
                         torch.device(DEV), torch.bfloat16)
    backend._pool = pool
    group = M.AttentionGroup(seq_indices=list(range(spec.num_seqs)), attention_type="decode_gpu",
                             cached_len_before=None, query_len=None, kv_len_after=t["kv_len"])
    meta = M.AttentionMetadata(groups=[group], decode_block_tables=t["block_tables"], block_size=16,
                               num_kv_heads=2, head_dim=64)
    ref = backend.decode_attention(0, t["query"], meta, pool)
    attn_out = torch.full((5 + spec.num_seqs, 14, 64), 7.0, dtype=torch.bfloat16, device=DEV)
    res = backend.decode_attention(0, t["query"], meta, pool, out=attn_out[5:])
    assert res.data_ptr() == attn_out[5:].data_ptr()
    assert torch.equal(attn_out[5:], ref) and (attn_out[:5] == 7.0).all()
