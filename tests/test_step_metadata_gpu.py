"""Per-step attention metadata on the device against the reference's
ModelInputBuilder (golden steps) and the oracle's restatement (GPU).

Integer outputs: bit-exact.  The decode tables and kv_len the builder
produces feed the decode kernel directly.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import mini_vllm_b200 as M
import oracle
from conftest import torch_to_np

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
KEYS = ["positions", "slot_mapping", "prefill_block_tables", "decode_block_tables", "sample_token_indices",
        "kv_len_after"]


def _outputs(md):
    return [md.positions, md.slot_mapping, md.prefill_block_tables, md.decode_block_tables,
            md.sample_token_indices, md.kv_len_after]


def _check(md, ref, name):
    for got, want, key in zip(_outputs(md), ref, KEYS):
        g = got.cpu().numpy().astype(np.int64)
        assert g.shape == want.shape and np.array_equal(g, want), (name, key)


def test_golden_steps_match_reference_builder(golden):
    cases, arrays = golden
    ran = 0
    for c in [c for c in cases if c["kind"] == "metadata"]:
        P = len(c["prefill"])
        prefill = [(c["block_lists"][i], c["cached"][i], c["query_len"][i], c["completes"][i]) for i in range(P)]
        decode = [(c["block_lists"][i], c["cached"][i]) for i in range(P, len(c["block_lists"]))]
        md = M.StepMetadataBuilder(c["block_size"], DEV).build(prefill, decode)
        _check(md, [arrays[f"{c['name']}/{k}"] for k in KEYS], c["name"])
        ran += 1
    assert ran >= 4


def _random_step(rng, n_prefill, n_decode, bs, nb):
    perm = rng.permutation(nb)
    pos = 0
    prefill, decode = [], []
    for _ in range(n_prefill):
        cached, q = int(rng.integers(0, 900)), int(rng.integers(1, 300))
        need = (cached + q + bs - 1) // bs
        prefill.append((perm[pos:pos + need].tolist(), cached, q, bool(rng.integers(0, 2))))
        pos += need
    for _ in range(n_decode):
        cached = int(rng.integers(0, 2047))
        need = (cached + 1 + bs - 1) // bs + int(rng.integers(0, 2))  # sometimes one spare block
        decode.append((perm[pos:pos + need].tolist(), cached))
        pos += need
    return prefill, decode


@pytest.mark.parametrize("n_prefill,n_decode,bs", [(0, 256, 16), (8, 256, 16), (3, 0, 8), (1, 1, 1)])
def test_random_steps_match_oracle(n_prefill, n_decode, bs):
    rng = np.random.default_rng(n_prefill * 1000 + n_decode + bs)
    prefill, decode = _random_step(rng, n_prefill, n_decode, bs, 200000)
    md = M.StepMetadataBuilder(bs, DEV).build(prefill, decode)
    lists = [p[0] for p in prefill] + [d[0] for d in decode]
    ref = oracle.step_metadata_numpy(lists, [p[1] for p in prefill] + [d[1] for d in decode],
                                     [p[2] for p in prefill] + [1] * len(decode), [p[3] for p in prefill],
                                     len(prefill), bs)
    _check(md, list(ref), f"{n_prefill}/{n_decode}/{bs}")


def test_position_without_block_raises():
    b = M.StepMetadataBuilder(16, DEV)
    with pytest.raises(RuntimeError, match="Block not allocated"):
        b.build([], [([3, 4], 32)])  # position 32 needs a third block
    md = b.build([], [([3, 4], 31)])  # the error word is clear afterwards
    assert md.slot_mapping.cpu().tolist() == [4 * 16 + 15]


def test_decode_runs_on_builder_outputs():
    """The decode tables and kv_len the builder produces drive the decode
    kernel: same result as the oracle decode over the same tables."""
    rng = np.random.default_rng(3)
    _, decode = _random_step(rng, 0, 64, 16, 20000)
    md = M.StepMetadataBuilder(16, DEV).build([], decode)
    g = torch.Generator().manual_seed(0)
    kc = torch.randn(20000, 2, 16, 64, generator=g).to(torch.bfloat16).to(DEV)
    vc = torch.randn(20000, 2, 16, 64, generator=g).to(torch.bfloat16).to(DEV)
    q = torch.randn(64, 14, 64, generator=g).to(torch.bfloat16).to(DEV)
    out = M.paged_decode_attention(q, kc, vc, md.decode_block_tables, md.decode_kv_len_after, 16)
    ref, st = oracle.decode(torch_to_np(q, "bf16"), torch_to_np(kc, "bf16"), torch_to_np(vc, "bf16"),
                            md.decode_block_tables.cpu().numpy(), md.decode_kv_len_after.cpu().numpy(), 16, "bf16")
    assert (st == 0).all()
    o = out.float().cpu().numpy()
    assert (np.abs(o - ref) <= 2e-3 + 1e-2 * np.abs(ref)).all()


def test_build_from_arrays_equals_list_build():
    """The padded-table entry point gives the same step as the list one."""
    rng = np.random.default_rng(9)
    prefill, decode = _random_step(rng, 4, 200, 16, 100000)
    lists = [p[0] for p in prefill] + [d[0] for d in decode]
    W = max(len(x) for x in lists) + 3
    tables = np.full((len(lists), W), -7, dtype=np.int64)  # junk past each row's count is never read
    for i, x in enumerate(lists):
        tables[i, :len(x)] = x
    b = M.StepMetadataBuilder(16, DEV)
    a = b.build(prefill, decode)
    c = b.build_from_arrays(tables, [len(x) for x in lists], [p[1] for p in prefill] + [d[1] for d in decode],
                            [p[2] for p in prefill] + [1] * len(decode), [p[3] for p in prefill], len(prefill))
    for x, y in zip(_outputs(a), _outputs(c)):
        assert torch.equal(x, y)
