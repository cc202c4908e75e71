"""Pin the CPU oracle to the reference (CPU only).

The golden vectors in tests/golden were produced by the reference's own
write_to_paged_cache, gather_paged_kv, AttentionBackendRef.decode_attention and
RotaryEmbedding (tests/golden/make_golden.py).  The C oracle must reproduce the writes and
gathers bit for bit and the decodes to float32 round-off; the numpy
restatement must agree with the C one.
"""

from __future__ import annotations

import numpy as np
import pytest

import make_golden as MG
import oracle


def _cases(golden, kind):
    cases, arrays = golden
    return [c for c in cases if c["kind"] == kind], arrays


def test_golden_fixture_covers_all_kinds(golden):
    cases, _ = golden
    kinds = {c["kind"] for c in cases}
    assert kinds == {"write", "write_spec", "gather", "decode", "decode_spec", "rope", "metadata"}
    assert len(cases) >= 60


@pytest.mark.parametrize("kind", ["write", "write_spec"])
def test_oracle_cache_write_bit_exact(golden, kind):
    cases, arrays = _cases(golden, kind)
    for c in cases:
        x = MG.write_inputs(c) if kind == "write" else MG.write_spec_inputs(c)
        assert MG.sha(x["kc0"], x["vc0"], x["key"], x["value"], x["slots"]) == c["inputs_sha256"], c["name"]
        bs = c.get("block_size") or x["block_size"]
        kc, vc = x["kc0"].copy(), x["vc0"].copy()
        if c.get("error"):
            with pytest.raises(IndexError, match="out of range"):
                oracle.cache_write(x["key"], x["value"], kc, vc, x["slots"], bs, c["dtype"])
        else:
            oracle.cache_write(x["key"], x["value"], kc, vc, x["slots"], bs, c["dtype"])
        # the whole pool — written rows and untouched rows — matches bit for bit
        assert MG.sha(kc, vc) == c["result_sha256"], c["name"]


def test_oracle_numpy_write_matches_reference(golden):
    cases, arrays = _cases(golden, "write")
    for c in cases:
        x = MG.write_inputs(c)
        kc, vc = x["kc0"].copy(), x["vc0"].copy()
        if c.get("error"):
            with pytest.raises(IndexError):
                oracle.cache_write_numpy(x["key"], x["value"], kc, vc, x["slots"], c["block_size"])
        else:
            oracle.cache_write_numpy(x["key"], x["value"], kc, vc, x["slots"], c["block_size"])
        assert MG.sha(kc, vc) == c["result_sha256"], c["name"]


def test_oracle_gather_matches_reference(golden):
    cases, arrays = _cases(golden, "gather")
    for c in cases:
        x = MG.gather_inputs(c)
        assert MG.sha(x["kc"], x["vc"], x["table"]) == c["inputs_sha256"]
        if c["error"]:
            with pytest.raises(IndexError, match="insufficient"):
                oracle.gather(x["kc"], x["vc"], x["table"], c["num_tokens"], c["block_size"], c["dtype"])
            continue
        k, v = oracle.gather(x["kc"], x["vc"], x["table"], c["num_tokens"], c["block_size"], c["dtype"])
        assert k.shape == arrays[f"{c['name']}/k"].shape
        assert np.array_equal(k, arrays[f"{c['name']}/k"]), c["name"]
        assert np.array_equal(v, arrays[f"{c['name']}/v"]), c["name"]


@pytest.mark.parametrize("kind", ["decode", "decode_spec"])
def test_oracle_decode_matches_reference(golden, kind):
    cases, arrays = _cases(golden, kind)
    for c in cases:
        x = MG.decode_inputs(c)
        assert MG.sha(x["q"], x["kc"], x["vc"], x["tables"], x["ctx"]) == c["inputs_sha256"], c["name"]
        out, status = oracle.decode(x["q"], x["kc"], x["vc"], x["tables"], x["ctx"], x["block_size"], c["dtype"])
        assert (status == oracle.ORACLE_OK).all(), c["name"]
        ref = arrays[f"{c['name']}/out"]
        # both sides see identical float32 inputs; the reference sums in fp32
        # (torch SDPA), the oracle in fp64 — round-off only
        np.testing.assert_allclose(out, ref, rtol=2e-5, atol=2e-5, err_msg=c["name"])


@pytest.mark.parametrize("kind", ["decode", "decode_spec"])
def test_oracle_c_and_numpy_restatements_agree(golden, kind):
    cases, _ = _cases(golden, kind)
    for c in cases:
        x = MG.decode_inputs(c)
        out, _ = oracle.decode(x["q"], x["kc"], x["vc"], x["tables"], x["ctx"], x["block_size"], c["dtype"])
        out_np = oracle.decode_numpy(x["q"], x["kc"], x["vc"], x["tables"], x["ctx"], x["block_size"], c["dtype"])
        np.testing.assert_allclose(out, out_np, rtol=1e-6, atol=1e-6, err_msg=c["name"])


def test_oracle_decode_error_statuses():
    q = np.zeros((3, 4, 64), np.float32)
    kc = np.zeros((4, 2, 16, 64), np.float32)
    tables = np.array([[0, -1], [1, -1], [7, -1]], np.int64)
    ctx = np.array([0, 40, 5], np.int32)
    _, st = oracle.decode(q, kc, kc, tables, ctx, 16, "f32")
    assert st.tolist() == [oracle.ORACLE_KV_LEN, oracle.ORACLE_TABLE_SHORT, oracle.ORACLE_BLOCK_ID]


def test_oracle_threads_do_not_change_results():
    from mini_vllm_b200 import workloads as W

    spec = W.make_spec(1, seed=5)
    t = W.numpy_tensors(spec, "bf16")
    a, _ = oracle.decode(t["query"], t["key_cache"], t["value_cache"], spec.block_tables, spec.context_lens, 16, "bf16", threads=1)
    b, _ = oracle.decode(t["query"], t["key_cache"], t["value_cache"], spec.block_tables, spec.context_lens, 16, "bf16", threads=0)
    assert np.array_equal(a, b)


def _storage(t, dtype):
    import torch

    if dtype == "bf16":
        return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return t.contiguous().numpy().copy()


def test_rope_tables_and_oracle_rope_write_bit_exact(golden):
    """rope_tables reproduces the reference's RotaryEmbedding cos/sin caches bit
    for bit (CPU), and the numpy restatement of rope followed by the oracle's
    write reproduces the reference's rotated q / k and the whole pool."""
    import mini_vllm_b200 as M

    cases, arrays = _cases(golden, "rope")
    assert len(cases) >= 5
    tdt = {"bf16": "bfloat16", "f16": "float16", "f32": "float32"}
    for c in cases:
        import torch

        dt = c["dtype"]
        x = MG.rope_inputs(c)
        assert MG.sha(x["q"], x["k"], x["v"], x["kc0"], x["vc0"], x["positions"], x["slots"]) == \
            c["inputs_sha256"], c["name"]
        cos, sin = M.rope_tables(c["head_dim"], c["theta"], c["max_seq"], getattr(torch, tdt[dt]))
        cos_np, sin_np = _storage(cos, dt), _storage(sin, dt)
        assert MG.sha(cos_np, sin_np) == c["tables_sha256"], c["name"]
        q_rot = oracle.rope_numpy(x["q"], x["positions"], cos_np, sin_np, dt)
        k_rot = oracle.rope_numpy(x["k"], x["positions"], cos_np, sin_np, dt)
        assert np.array_equal(q_rot, arrays[f"{c['name']}/q_rot"]), c["name"]
        assert np.array_equal(k_rot, arrays[f"{c['name']}/k_rot"]), c["name"]
        kc, vc = x["kc0"].copy(), x["vc0"].copy()
        oracle.cache_write(k_rot, x["v"], kc, vc, x["slots"], c["block_size"], dt)
        assert MG.sha(kc, vc) == c["result_sha256"], c["name"]


def test_oracle_step_metadata_matches_reference_builder(golden):
    """The numpy restatement of ModelInputBuilder.build reproduces the
    reference's positions, slot mapping, padded tables, sample indices and
    kv_len_after for every golden step."""
    cases, arrays = _cases(golden, "metadata")
    assert len(cases) >= 4
    for c in cases:
        P = len(c["prefill"])
        out = oracle.step_metadata_numpy(c["block_lists"], c["cached"], c["query_len"], c["completes"], P,
                                         c["block_size"])
        for got, key in zip(out, ["positions", "slot_mapping", "prefill_block_tables", "decode_block_tables",
                                  "sample_token_indices", "kv_len_after"]):
            ref = arrays[f"{c['name']}/{key}"]
            assert got.shape == ref.shape and np.array_equal(got, ref), (c["name"], key)
