"""The config-5 harness on the CPU: a random Qwen2 checkpoint and its id
tokenizer load through the reference's own loaders, and the reference's
LLMEngine (its torch "reference" backend, device cpu) serves requests from
it; the "b200" branch is added to AttentionBackend.create without changing
any other name.  The GPU comparison is tests/test_engine_dropin_gpu.py."""

from __future__ import annotations

import os
import tempfile

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
pytestmark = pytest.mark.skipif(not os.path.isdir(os.path.join(REPO, "baseline", "_ref", "mini_vllm")),
                                reason="the reference is not installed in baseline/_ref")


def test_random_checkpoint_serves_on_the_reference_engine():
    from mini_vllm_b200 import reference_engine as RE

    d = tempfile.mkdtemp(prefix="mvb_qwen2_cpu_")
    cfg = RE.write_random_checkpoint(d, num_layers=2, vocab_size=512, seed=1)
    assert cfg["hidden_size"] == 896 and cfg["num_attention_heads"] == 14 and cfg["num_key_value_heads"] == 2
    RE.register_backend()
    from mini_vllm.config import Config
    from mini_vllm.engine.engine import LLMEngine
    from mini_vllm.model_runner.config_adapter import ConfigAdapter

    mc = ConfigAdapter.from_pretrained(d)
    assert (mc.num_layers, mc.head_dim, mc.rope_theta) == (2, 64, 1e6)
    c = Config(executor_type="paged", attention_backend="reference", model_path=d, device="cpu", block_size=16,
               num_gpu_blocks=64, max_num_seqs=4, max_num_batched_tokens=256, max_num_prefill_tokens=256,
               max_prefill_chunk_size=64, print_step_events=False, enable_prefix_caching=False)
    eng = LLMEngine(c)
    assert eng._executor.tokenize(RE.prompt_text([5, 17, 300])) == [5, 17, 300]
    g = torch.Generator().manual_seed(0)
    for n in (20, 37):
        eng.add_request(RE.prompt_text(torch.randint(0, 512, (n,), generator=g).tolist()), max_new_tokens=4)
    outs = eng.run_until_done()
    assert len(outs) == 2 and all(len(v.split()) == 4 for v in outs.values())


def test_b200_branch_leaves_other_names_alone():
    from mini_vllm_b200 import reference_engine as RE

    RE.register_backend()
    from mini_vllm.attention.backend import AttentionBackend
    from mini_vllm.attention.paged_attention_ref import AttentionBackendRef
    from mini_vllm.model_runner.base import ModelConfig

    mc = ModelConfig(num_heads=14, num_kv_heads=2, head_dim=64)
    assert isinstance(AttentionBackend.create(mc, backend="reference"), AttentionBackendRef)
    with pytest.raises(ValueError, match="Unknown AttentionBackend"):
        AttentionBackend.create(mc, backend="nope")
