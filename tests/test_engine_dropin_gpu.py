"""The B200 backend inside the reference's own engine (GPU).

The reference (installed in baseline/_ref by baseline/install_reference.sh) runs
unchanged: ``LLMEngine`` -> ``EngineCore.step`` -> ``Scheduler`` /
``BlockManager`` / ``ModelInputBuilder`` -> ``PagedExecutor`` ->
``QwenModelRunner.execute_model`` (mini_vllm/model_runner/qwen_runner.py:
163-190), which calls ``write_kv_cache``, ``prefill_attention`` and
``decode_attention`` of the backend that ``AttentionBackend.create`` returns
for ``Config.attention_backend``.  ``register_backend`` adds the ``"b200"``
branch to that factory; everything else is the reference's code.

A random Qwen2 checkpoint (Qwen2-0.5B widths — hidden 896, 14 / 2 heads of
64, MLP 4864, RoPE theta 1e6 — with 2 layers and an 8192-token vocabulary to
keep the test short; weights ~ N(0, 0.02)) serves the same requests on two
engines, one with the reference's torch backend ("reference") and one with
"b200".  Chunked prefill (64-token chunks over prompts of up to 300 tokens)
reads cached prefixes through the gather kernel, and every decode step runs
the kernel the plan picks for its batch.  Every step's logits must agree within
LOGIT_ATOL row by row (rows are sequences), and the greedy tokens must agree
wherever the reference's top-2 margin exceeds twice that bound.  Where the
margin is smaller (a near-tie: random weights make logits of ~8k tokens
close), the two engines may sample different tokens; that sequence then
continues from a different token in each engine, and its later rows are no
longer compared.
"""

from __future__ import annotations

import os
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# max |logit difference|: the model runs in fp16 (the reference's ConfigAdapter),
# whose rounding of logits of magnitude ~1-3 is ~1e-3; attention outputs agree to
# 2e-3 + 1e-2 |ref| (the decode parity bound), which two layers carry to the
# logits at the 1e-2 level at most
LOGIT_ATOL = 3e-2


def _have_reference() -> bool:
    return os.path.isdir(os.path.join(REPO, "baseline", "_ref", "mini_vllm"))


@pytest.fixture(scope="module")
def checkpoint():
    if not _have_reference():
        pytest.skip("the reference is not installed in baseline/_ref (baseline/install_reference.sh)")
    from mini_vllm_b200 import reference_engine as RE

    d = tempfile.mkdtemp(prefix="mvb_qwen2_")
    RE.write_random_checkpoint(d, num_layers=2, vocab_size=8192, seed=5)
    return d


def _run_engine(model_path: str, backend: str, prompts, max_new_tokens: int):
    from mini_vllm_b200 import reference_engine as RE

    RE.register_backend(overlap_after_write=True)
    from mini_vllm.config import Config
    from mini_vllm.engine.engine import LLMEngine

    cfg = Config(executor_type="paged", attention_backend=backend, model_path=model_path, device="cuda",
                 block_size=16, num_gpu_blocks=256, max_num_seqs=8, max_num_batched_tokens=512,
                 max_num_prefill_tokens=512, max_prefill_chunk_size=64, print_step_events=False,
                 enable_prefix_caching=False)
    eng = LLMEngine(cfg)
    runner = eng._executor._model_runner
    logits = []
    inner = runner.execute_model

    def record(model_input):
        out = inner(model_input)
        logits.append((out.float().cpu(), _sampled_ids(model_input)))
        return out

    runner.execute_model = record
    for ids in prompts:
        eng.add_request(RE.prompt_text(ids), max_new_tokens=max_new_tokens)
    outputs = eng.run_until_done()
    return outputs, logits, type(eng._executor._attention_backend).__name__


def _sampled_ids(model_input):
    """The sequence of each logits row: the sequences with a sample index, in order."""
    return [info.sequence_id for info in model_input.sequence_info if info.sample_output_index is not None]


def test_engine_logits_match_the_reference_backend(checkpoint):
    g = torch.Generator().manual_seed(11)
    lens = [17, 300, 64, 129, 5, 250]
    prompts = [torch.randint(0, 8192, (n,), generator=g).tolist() for n in lens]
    ref_out, ref_logits, ref_cls = _run_engine(checkpoint, "reference", prompts, 12)
    b2_out, b2_logits, b2_cls = _run_engine(checkpoint, "b200", prompts, 12)
    assert ref_cls == "AttentionBackendRef" and b2_cls == "AttentionBackendB200"
    assert len(ref_logits) == len(b2_logits) > 12  # prefill chunks, then decode steps
    worst, compared, diverged = 0.0, 0, set()
    for step, ((a, ids_a), (b, ids_b)) in enumerate(zip(ref_logits, b2_logits)):
        assert ids_a == ids_b and a.shape == b.shape, step
        assert torch.isfinite(b).all(), step
        for row, sid in enumerate(ids_a):
            if sid in diverged:
                continue
            d = (a[row] - b[row]).abs().max().item()
            worst = max(worst, d)
            compared += 1
            assert d <= LOGIT_ATOL, f"step {step} sequence {sid}: max |logit diff| {d:.3e}"
            if a[row].argmax() != b[row].argmax():
                top2 = a[row].topk(2).values
                assert top2[0] - top2[1] <= 2 * LOGIT_ATOL, f"step {step} sequence {sid}: tokens differ"
                diverged.add(sid)  # a near-tie: the engines continue from different tokens
    assert compared > 40 and len(diverged) <= 2
    assert sorted(ref_out) == sorted(b2_out)
    print(f"engine drop-in: {len(ref_logits)} steps, {compared} rows compared, max |logit diff| {worst:.3e}, "
          f"near-tie divergences {len(diverged)}")


def test_unknown_backend_still_raises(checkpoint):
    from mini_vllm_b200 import reference_engine as RE

    RE.register_backend()
    from mini_vllm.attention.backend import AttentionBackend
    from mini_vllm.model_runner.base import ModelConfig

    with pytest.raises(ValueError, match="Unknown AttentionBackend"):
        AttentionBackend.create(ModelConfig(num_heads=14, num_kv_heads=2, head_dim=64), backend="nope")
