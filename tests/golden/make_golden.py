"""Generate the golden vectors that pin the CPU oracle to the reference.

Run in a container that has the reference checkout (read-only) on disk:

    python tests/golden/make_golden.py [/path/to/reference]

It imports the reference's own torch implementation of the path —
``write_to_paged_cache`` (mini_vllm/cache/cache_write.py:25-74),
``gather_paged_kv`` (mini_vllm/cache/cache_read.py:19-84) and
``AttentionBackendRef.decode_attention``
(mini_vllm/attention/paged_attention_ref.py:102-161) — runs it on seeded
inputs, and writes ``golden.npz`` + ``golden.json`` next to this file.

The fixture holds outputs only.  Every case's inputs are rebuilt by the
``*_inputs`` functions below from the parameters recorded in ``golden.json``
(numpy's PCG64 streams are stable across machines), and the recorded SHA-256
of those inputs proves a rebuild is identical.  Write results are stored as
SHA-256 of the whole resulting caches (a bit-exact check) plus the rows the
write touched.  The tests import this module for the ``*_inputs`` builders
only; nothing here touches the reference unless ``main`` runs.

bf16 / f16 decode inputs are upcast to float32 before the reference runs, so
the reference accumulates in fp32 ("fp32 accumulation on both sides").
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from typing import Dict, List, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

from mini_vllm_b200 import workloads as W  # noqa: E402


def sha(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def _conv(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return W.f32_to_bf16_bits(x.astype(np.float32))
    return x.astype(np.float16 if dtype == "f16" else np.float32)


def ramp(shape, base: float, dtype: str) -> np.ndarray:
    """flat[i] = base + i in the storage type — the reference GPU tests'
    deterministic inputs (test_paged_attention_gpu.py:118-124)."""
    x = (base + np.arange(int(np.prod(shape)), dtype=np.float64)).reshape(shape)
    return _conv(x, dtype)


# ---------------------------------------------------------------------------
# deterministic case inputs (shared with the tests)
# ---------------------------------------------------------------------------
def write_inputs(c: Dict) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(c["seed"])
    nb, kh, bs, d = c["num_blocks"], c["num_kv_heads"], c["block_size"], c["head_dim"]
    t = len(c["slots"])
    kc0 = _conv(rng.standard_normal((nb, kh, bs, d), dtype=np.float32), c["dtype"])
    vc0 = _conv(rng.standard_normal((nb, kh, bs, d), dtype=np.float32), c["dtype"])
    if c.get("init") == "zeros":
        kc0[...] = 0
        vc0[...] = 0
    key = _conv(rng.standard_normal((t, kh, d), dtype=np.float32), c["dtype"])
    value = _conv(rng.standard_normal((t, kh, d), dtype=np.float32), c["dtype"])
    return {"kc0": kc0, "vc0": vc0, "key": key, "value": value,
            "slots": np.asarray(c["slots"], dtype=np.int64)}


def gather_inputs(c: Dict) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(c["seed"])
    shape = (c["num_blocks"], c["num_kv_heads"], c["block_size"], c["head_dim"])
    return {"kc": _conv(rng.standard_normal(shape, dtype=np.float32), c["dtype"]),
            "vc": _conv(rng.standard_normal(shape, dtype=np.float32), c["dtype"]),
            "table": np.asarray(c["table"], dtype=np.int64)}


def decode_inputs(c: Dict) -> Dict[str, np.ndarray]:
    """Inputs of a decode case: either a workloads config or an explicit table."""
    if c["kind"] == "decode_spec":
        spec = W.make_spec(c["config"], seed=c["seed"], num_seqs=c.get("num_seqs"))
        t = W.numpy_tensors(spec, c["dtype"])
        return {"q": t["query"], "kc": t["key_cache"], "vc": t["value_cache"],
                "tables": spec.block_tables, "ctx": spec.context_lens.astype(np.int32),
                "block_size": spec.block_size}
    nb, h, kh, bs, d = c["num_blocks"], c["num_heads"], c["num_kv_heads"], c["block_size"], c["head_dim"]
    nseq = len(c["ctx"])
    if c.get("values") == "ramp":
        q = ramp((nseq, h, d), 50.0, c["dtype"])
        kc = ramp((nb, kh, bs, d), 10.0, c["dtype"])
        vc = ramp((nb, kh, bs, d), 1000.0, c["dtype"])
    else:
        rng = np.random.default_rng(c["seed"])
        q = _conv(rng.standard_normal((nseq, h, d), dtype=np.float32), c["dtype"])
        kc = _conv(rng.standard_normal((nb, kh, bs, d), dtype=np.float32), c["dtype"])
        vc = _conv(rng.standard_normal((nb, kh, bs, d), dtype=np.float32), c["dtype"])
    return {"q": q, "kc": kc, "vc": vc, "tables": np.asarray(c["tables"], dtype=np.int64),
            "ctx": np.asarray(c["ctx"], dtype=np.int32), "block_size": bs}


def write_spec_inputs(c: Dict) -> Dict[str, np.ndarray]:
    spec = W.make_spec(c["config"], seed=c["seed"])
    t = W.numpy_tensors(spec, c["dtype"])
    return {"kc0": t["key_cache"], "vc0": t["value_cache"], "key": t["new_key"],
            "value": t["new_value"], "slots": spec.slot_mapping, "block_size": spec.block_size}


def rope_inputs(c: Dict) -> Dict[str, np.ndarray]:
    """Inputs of a fused RoPE + write case (query, key, value, positions, pools, slots)."""
    rng = np.random.default_rng(c["seed"])
    t, h, kh, d = c["num_tokens"], c["num_heads"], c["num_kv_heads"], c["head_dim"]
    nb, bs, dt = c["num_blocks"], c["block_size"], c["dtype"]
    slots = rng.permutation(nb * bs)[:t].astype(np.int64)
    for i in c.get("skip", []):
        slots[i] = -1
    lo = c.get("pos_min", 0)
    return {"q": _conv(rng.standard_normal((t, h, d), dtype=np.float32), dt),
            "k": _conv(rng.standard_normal((t, kh, d), dtype=np.float32), dt),
            "v": _conv(rng.standard_normal((t, kh, d), dtype=np.float32), dt),
            "kc0": _conv(rng.standard_normal((nb, kh, bs, d), dtype=np.float32), dt),
            "vc0": _conv(rng.standard_normal((nb, kh, bs, d), dtype=np.float32), dt),
            "positions": rng.integers(lo, c["max_seq"], size=t).astype(np.int64),
            "slots": slots}


# ---------------------------------------------------------------------------
# case list
# ---------------------------------------------------------------------------
def case_list() -> List[Dict]:
    cases: List[Dict] = []

    def w(name, dtype, nb, kh, bs, d, slots, seed, error=False, init="random"):
        cases.append(dict(kind="write", name=name, dtype=dtype, num_blocks=nb, num_kv_heads=kh,
                          block_size=bs, head_dim=d, slots=slots, seed=seed, expect_error=error,
                          init=init))

    for dt in ("f16", "bf16", "f32"):
        # the reference's test_cache_write.py scenarios (pool 4 x 2 x 4 x 8)
        w(f"w_single_{dt}", dt, 4, 2, 4, 8, [5], 1)
        w(f"w_prefill_{dt}", dt, 4, 2, 4, 8, list(range(8)), 2)
        w(f"w_batched_{dt}", dt, 4, 2, 4, 8, [0, 12], 3)
        w(f"w_boundary_{dt}", dt, 4, 2, 4, 8, [3, 4, 7, 8], 4)
        w(f"w_noncontig_{dt}", dt, 32, 2, 4, 8, [20, 69, 14], 5)
        w(f"w_dup_lastwins_{dt}", dt, 4, 2, 4, 8, [5, 5], 6)
        w(f"w_skip_{dt}", dt, 4, 2, 4, 8, [-1, 5, -1, 8], 7, init="zeros")
        w(f"w_oob_{dt}", dt, 4, 2, 4, 8, [16], 8, error=True)
        w(f"w_lt_minus1_{dt}", dt, 4, 2, 4, 8, [-2], 9, error=True)
        w(f"w_partial_oob_{dt}", dt, 4, 2, 4, 8, [1, 2, 99, 3], 10, error=True)
        # GPU-kernel shapes
        w(f"w_d64_{dt}", dt, 64, 2, 16, 64, [0, 17, 33, 50, 99, 1023], 11)
        w(f"w_d128_{dt}", dt, 8, 8, 16, 128, [5, 100, 127, 16, 17], 12)
    for dt in ("f32", "bf16"):
        cases.append(dict(kind="write_spec", name=f"w_cfg1_{dt}", dtype=dt, config=1, seed=0))

    def g(name, dtype, nb, kh, bs, d, table, n, seed, error=False):
        cases.append(dict(kind="gather", name=name, dtype=dtype, num_blocks=nb, num_kv_heads=kh,
                          block_size=bs, head_dim=d, table=table, num_tokens=n, seed=seed,
                          expect_error=error))

    # the reference's test_paged_attention_ref.py gather scenarios (8/2/32, BS 4)
    g("g_full_block", "f16", 32, 2, 4, 32, [3], 4, 20)
    g("g_partial", "f16", 32, 2, 4, 32, [3], 3, 21)
    g("g_multi", "f16", 32, 2, 4, 32, [1, 2, 3], 10, 22)
    g("g_noncontig", "bf16", 32, 2, 4, 32, [7, 3, 15], 10, 23)
    g("g_zero", "f32", 32, 2, 4, 32, [], 0, 24)
    g("g_insufficient", "f32", 32, 2, 4, 32, [0], 8, 25, error=True)
    g("g_d64_bs16", "bf16", 64, 2, 16, 64, [10, 50], 19, 26)

    def ds(name, config, seed, dt, num_seqs=None):
        cases.append(dict(kind="decode_spec", name=name, dtype=dt, config=config, seed=seed,
                          num_seqs=num_seqs))

    ds("d_cfg1_f32_s0", 1, 0, "f32")
    ds("d_cfg1_f32_s1", 1, 1, "f32")
    ds("d_cfg1_bf16_s0", 1, 0, "bf16")
    ds("d_cfg1_f16_s2", 1, 2, "f16")
    ds("d_cfg2_bf16_16seq", 2, 3, "bf16", num_seqs=16)
    ds("d_cfg4_bf16_8seq", 4, 4, "bf16", num_seqs=8)

    def dt_(name, dtype, nb, h, kh, bs, d, tables, ctx, seed, values="random"):
        cases.append(dict(kind="decode", name=name, dtype=dtype, num_blocks=nb, num_heads=h,
                          num_kv_heads=kh, block_size=bs, head_dim=d, tables=tables, ctx=ctx,
                          seed=seed, values=values))

    # the reference oracle tests' shape (test_paged_attention_ref.py:26-31: 8 q / 2 KV / D 32, BS 4)
    dt_("d_ref_single", "f16", 32, 8, 2, 4, 32, [[0, 1, -1]], [5], 30)
    dt_("d_ref_multi", "f16", 32, 8, 2, 4, 32, [[0, 1, -1, -1], [4, 5, 6, -1], [8, 9, 10, 11]],
        [5, 9, 13], 31)
    dt_("d_ref_noncontig", "f16", 32, 8, 2, 4, 32, [[7, 3, 5]], [9], 32)
    # the reference GPU tests' shape (4 q / 2 KV / D 64, BS 16) with ramp values
    dt_("d_gpu_ramp_ragged", "f16", 16, 4, 2, 16, 64,
        [[0, -1], [1, -1], [2, -1], [3, -1], [4, -1], [5, 6], [7, 8], [9, 10]],
        [1, 3, 7, 15, 16, 17, 31, 32], 33, values="ramp")
    dt_("d_gpu_ramp_noncontig", "f16", 16, 4, 2, 16, 64, [[10, 5]], [19], 34, values="ramp")
    dt_("d_gpu_qwen8q", "bf16", 8, 8, 2, 16, 64, [[0, -1], [3, 6]], [8, 24], 35)
    dt_("d_gqa7_d64_bf16", "bf16", 16, 14, 2, 16, 64, [[5, 9, 1, -1], [15, 2, 3, 4], [7, -1, -1, -1]],
        [40, 64, 1], 36)
    dt_("d_gqa4_d128_bf16", "bf16", 12, 32, 8, 16, 128, [[5, 9, 1, -1], [11, 2, 3, 4]], [33, 49], 37)
    dt_("d_bs32_f16", "f16", 12, 4, 2, 32, 64, [[3, 9, -1], [1, 2, 0]], [40, 96], 38)
    dt_("d_gqa7_d64_f32", "f32", 16, 14, 2, 16, 64, [[4, 8, 0], [14, 1, 2]], [48, 33], 39)

    def r(name, dtype, t, h, kh, d, theta, max_seq, nb, bs, seed, **kw):
        cases.append(dict(kind="rope", name=name, dtype=dtype, num_tokens=t, num_heads=h, num_kv_heads=kh,
                          head_dim=d, theta=theta, max_seq=max_seq, num_blocks=nb, block_size=bs, seed=seed,
                          **kw))

    # RotaryEmbedding + write_to_paged_cache, as the runner applies them (qwen_runner.py:163-170)
    r("r_qwen_bf16", "bf16", 16, 14, 2, 64, 1e6, 4096, 16, 16, 40, skip=[3])
    r("r_d128_f16", "f16", 7, 8, 4, 128, 1e4, 512, 8, 16, 41)
    r("r_small_f32", "f32", 5, 4, 2, 64, 1e6, 64, 4, 4, 42, skip=[0])
    r("r_far_pos_bf16", "bf16", 9, 4, 1, 64, 1e6, 32768, 4, 16, 43, pos_min=30000)
    r("r_d32_bf16", "bf16", 3, 2, 1, 32, 1e4, 128, 2, 4, 44)

    def m(name, bs, nblocks, chunk, prefill, decode, seed):
        cases.append(dict(kind="metadata", name=name, dtype="i64", block_size=bs, num_gpu_blocks=nblocks,
                          chunk=chunk, prefill=prefill, decode=decode, seed=seed))

    # ModelInputBuilder.build steps: (prompt_len, prefill_cursor) / (prompt_len, generated)
    m("m_mixed_bs4", 4, 64, 4, [[10, 0], [10, 4], [9, 8]], [[6, 1], [7, 2], [9, 3], [5, 1]], 50)
    m("m_chunked_bs16", 16, 256, 128, [[300, 64], [40, 0]], [[100, 5], [16, 1]], 51)
    m("m_decode32_bs16", 16, 2048, 64, [], [[int(x), int(g)] for x, g in
                                              zip(np.random.default_rng(52).integers(100, 900, 32),
                                                  np.random.default_rng(53).integers(1, 40, 32))], 52)
    m("m_prefill_only_bs8", 8, 128, 32, [[70, 0], [70, 32]], [], 53)
    return cases


# ---------------------------------------------------------------------------
# reference runs
# ---------------------------------------------------------------------------
def main(ref_root: str) -> None:
    import torch

    sys.path.insert(0, ref_root)
    from mini_vllm.attention.paged_attention_ref import AttentionBackendRef
    from mini_vllm.cache.cache_read import gather_paged_kv
    from mini_vllm.cache.cache_write import write_to_paged_cache
    from mini_vllm.cache.pool import KVCachePool
    from mini_vllm.cache.allocator import BlockAllocator
    from mini_vllm.cache.manager import BlockManager
    from mini_vllm.config import Config
    from mini_vllm.engine.input_builder import ModelInputBuilder
    from mini_vllm.model.rotary import RotaryEmbedding
    from mini_vllm.sequence.sampling_params import SamplingParams
    from mini_vllm.sequence.sequence import Sequence
    from mini_vllm.sequence.status import Status
    from mini_vllm.model_runner.base import AttentionGroup, AttentionMetadata, ModelConfig

    def to_torch(a: np.ndarray, dtype: str) -> torch.Tensor:
        if dtype == "bf16":
            return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
        return torch.from_numpy(a.copy())

    def to_numpy(t: torch.Tensor, dtype: str) -> np.ndarray:
        if dtype == "bf16":
            return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
        return t.contiguous().numpy().copy()

    def up32(a: np.ndarray, dtype: str) -> torch.Tensor:
        if dtype == "bf16":
            return torch.from_numpy((a.astype(np.uint32) << 16).view(np.float32))
        return torch.from_numpy(a.astype(np.float32))

    arrays: Dict[str, np.ndarray] = {}
    cases = case_list()
    for c in cases:
        name, dt = c["name"], c["dtype"]
        if c["kind"] in ("write", "write_spec"):
            x = write_inputs(c) if c["kind"] == "write" else write_spec_inputs(c)
            bs = c.get("block_size") or x["block_size"]
            kc, vc = to_torch(x["kc0"], dt), to_torch(x["vc0"], dt)
            err = None
            try:
                write_to_paged_cache(to_torch(x["key"], dt), to_torch(x["value"], dt), kc, vc,
                                     torch.from_numpy(x["slots"]), bs)
            except IndexError as e:
                err = f"IndexError: {e}"
            if c["kind"] == "write":
                assert (err is not None) == c["expect_error"], (name, err)
            c["error"] = err
            c["inputs_sha256"] = sha(x["kc0"], x["vc0"], x["key"], x["value"], x["slots"])
            c["result_sha256"] = sha(to_numpy(kc, dt), to_numpy(vc, dt))
            # rows the write touched (the oracle's last-writer-wins content)
            rows_k, rows_v = [], []
            for s in x["slots"].tolist():
                if 0 <= s < kc.shape[0] * bs:
                    rows_k.append(to_numpy(kc[s // bs, :, s % bs, :], dt))
                    rows_v.append(to_numpy(vc[s // bs, :, s % bs, :], dt))
            if rows_k:
                arrays[f"{name}/rows_k"] = np.stack(rows_k)
                arrays[f"{name}/rows_v"] = np.stack(rows_v)
        elif c["kind"] == "metadata":
            rng = np.random.default_rng(c["seed"])
            cfg = Config(block_size=c["block_size"], num_gpu_blocks=c["num_gpu_blocks"],
                         max_prefill_chunk_size=c["chunk"], max_num_seqs=1024, max_num_batched_tokens=1 << 20,
                         vocab_size=1 << 16, device="cpu")
            mgr = BlockManager(c["block_size"], BlockAllocator(num_blocks=c["num_gpu_blocks"]))
            seqs_p, seqs_d = [], []
            for i, (plen, cursor) in enumerate(c["prefill"]):
                sq = Sequence(f"p{i}", f"gp{i}", rng.integers(0, 1 << 16, plen).tolist(),
                              SamplingParams(max_tokens=1 << 12), 0.0)
                sq.prefill_cursor = cursor
                sq.status = Status.PREFILL
                seqs_p.append(sq)
            for i, (plen, gen) in enumerate(c["decode"]):
                sq = Sequence(f"d{i}", f"gd{i}", rng.integers(0, 1 << 16, plen).tolist(),
                              SamplingParams(max_tokens=1 << 12), 0.0)
                sq.prefill_cursor = plen
                sq.status = Status.RUNNING
                sq.output_token_ids = [7] * gen
                sq.num_generated_tokens = gen
                seqs_d.append(sq)
            # positions each sequence needs blocks for, allocated position-major so that
            # the sequences' blocks interleave in the pool
            need = [min(len(sq.prompt_token_ids), sq.prefill_cursor + c["chunk"]) for sq in seqs_p] + \
                   [len(sq.prompt_token_ids) + sq.num_generated_tokens for sq in seqs_d]
            for sq in seqs_p + seqs_d:
                mgr.allocate_for_seq(sq)
            for pos in range(max(need, default=0)):
                for sq, n in zip(seqs_p + seqs_d, need):
                    if pos < n:
                        mgr.ensure_block(sq, pos)
            mi = ModelInputBuilder(mgr, cfg).build(seqs_p, seqs_d)
            c["block_lists"] = [mgr.get_block_table(sq.seq_id) for sq in seqs_p + seqs_d]
            groups = {g.attention_type: g for g in mi.attn_metadata.groups}
            c["cached"] = [int(x) for g in mi.attn_metadata.groups for x in g.cached_len_before.tolist()]
            c["query_len"] = [int(x) for g in mi.attn_metadata.groups for x in g.query_len.tolist()]
            c["completes"] = [sq.prefill_cursor + min(c["chunk"], len(sq.prompt_token_ids) - sq.prefill_cursor)
                              >= len(sq.prompt_token_ids) for sq in seqs_p]
            assert [g.attention_type for g in mi.attn_metadata.groups] == \
                (["prefill_gpu"] if seqs_p else []) + (["decode_gpu"] if seqs_d else []), groups.keys()
            arrays[f"{name}/positions"] = mi.positions.numpy()
            arrays[f"{name}/slot_mapping"] = mi.slot_mapping.numpy()
            arrays[f"{name}/prefill_block_tables"] = mi.attn_metadata.prefill_block_tables.numpy()
            arrays[f"{name}/decode_block_tables"] = mi.attn_metadata.decode_block_tables.numpy()
            arrays[f"{name}/sample_token_indices"] = mi.sample_token_indices.numpy()
            arrays[f"{name}/kv_len_after"] = np.concatenate(
                [g.kv_len_after.numpy() for g in mi.attn_metadata.groups]) if mi.attn_metadata.groups \
                else np.zeros(0, np.int64)
        elif c["kind"] == "rope":
            x = rope_inputs(c)
            c["inputs_sha256"] = sha(x["q"], x["k"], x["v"], x["kc0"], x["vc0"], x["positions"], x["slots"])
            tdt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[dt]
            rope = RotaryEmbedding(head_dim=c["head_dim"], theta=c["theta"], max_seq_len=c["max_seq"], dtype=tdt)
            c["tables_sha256"] = sha(to_numpy(rope.cos, dt), to_numpy(rope.sin, dt))
            pos = torch.from_numpy(x["positions"])
            q_rot = rope(to_torch(x["q"], dt), pos)
            k_rot = rope(to_torch(x["k"], dt), pos)
            kc, vc = to_torch(x["kc0"], dt), to_torch(x["vc0"], dt)
            write_to_paged_cache(k_rot, to_torch(x["v"], dt), kc, vc, torch.from_numpy(x["slots"]),
                                 c["block_size"])
            arrays[f"{name}/q_rot"], arrays[f"{name}/k_rot"] = to_numpy(q_rot, dt), to_numpy(k_rot, dt)
            c["result_sha256"] = sha(to_numpy(kc, dt), to_numpy(vc, dt))
        elif c["kind"] == "gather":
            x = gather_inputs(c)
            c["inputs_sha256"] = sha(x["kc"], x["vc"], x["table"])
            err = None
            try:
                k, v = gather_paged_kv(to_torch(x["kc"], dt), to_torch(x["vc"], dt),
                                       x["table"].tolist(), c["num_tokens"], c["block_size"])
                arrays[f"{name}/k"], arrays[f"{name}/v"] = to_numpy(k, dt), to_numpy(v, dt)
            except IndexError as e:
                err = f"IndexError: {e}"
            assert (err is not None) == c["expect_error"], (name, err)
            c["error"] = err
        else:
            x = decode_inputs(c)
            c["inputs_sha256"] = sha(x["q"], x["kc"], x["vc"], x["tables"], x["ctx"])
            q, kcf, vcf = up32(x["q"], dt), up32(x["kc"], dt), up32(x["vc"], dt)
            nd, kh, bs = q.shape[0], kcf.shape[1], x["block_size"]
            cached = torch.from_numpy(x["ctx"].astype(np.int64) - 1)
            group = AttentionGroup(seq_indices=list(range(nd)), attention_type="decode_gpu",
                                   cached_len_before=cached, query_len=torch.ones(nd, dtype=torch.long),
                                   kv_len_after=cached + 1)
            meta = AttentionMetadata(groups=[group], decode_block_tables=torch.from_numpy(x["tables"]),
                                     block_size=bs, num_kv_heads=kh, head_dim=q.shape[2])
            pool = KVCachePool(key_caches=[kcf], value_caches=[vcf], num_blocks=kcf.shape[0],
                               block_size=bs, num_layers=1, num_kv_heads=kh, head_dim=q.shape[2],
                               device=torch.device("cpu"), dtype=torch.float32)
            be = AttentionBackendRef(ModelConfig(num_kv_heads=kh, head_dim=q.shape[2]))
            be._pool = pool
            arrays[f"{name}/out"] = be.decode_attention(0, q, meta, pool).numpy().astype(np.float32)

    np.savez_compressed(os.path.join(HERE, "golden.npz"), **arrays)
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump({"generator": "tests/golden/make_golden.py", "reference_torch": torch.__version__,
                   "cases": cases}, f, indent=1)
    print(f"{len(cases)} cases, {sum(a.nbytes for a in arrays.values()) / 1e6:.3f} MB raw")


def load_golden():
    with open(os.path.join(HERE, "golden.json")) as f:
        meta = json.load(f)
    arrays = dict(np.load(os.path.join(HERE, "golden.npz")))
    return meta["cases"], arrays


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
