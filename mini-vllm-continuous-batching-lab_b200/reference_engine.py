"""Run the reference's engine (mini_vllm) on this backend.

The reference selects its attention plug-in in ``AttentionBackend.create``
(mini_vllm/attention/backend.py:98-113) from ``Config.attention_backend``
(mini_vllm/config.py:76), through ``PagedExecutor`` (executor/paged_executor.py:
47-49).  ``register_backend`` adds the ``"b200"`` branch to that factory at run
time — the same one branch a maintainer would add to the file — so
``LLMEngine(Config(executor_type="paged", attention_backend="b200", ...))``
runs the reference's scheduler, block manager, input builder, Qwen model
runner and engine step loop unchanged, with every KV write, decode and prefill
attention call on the B200 kernels.

``write_random_checkpoint`` writes a Qwen2-shaped model directory the
reference's loaders read (``config.json`` for ConfigAdapter, ``model.safetensors``
in the Hugging Face key layout for load_qwen_weights, and a tokenizer for
PagedExecutor): weights ~ N(0, 0.02), RMSNorm weights 1, no network and no
real checkpoint needed.  Its tokenizer is a word-level map of the decimal
token ids ("17 4096 3" -> [17, 4096, 3]), so synthetic prompts are sequences
of ids drawn from the vocabulary.

The reference itself is not part of this package: it is installed separately
(``baseline/install_reference.sh`` puts it in ``baseline/_ref``);
``import_reference`` puts that directory on ``sys.path``.
"""

from __future__ import annotations

import json
import os
import sys
from typing import Any, Dict, Optional

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE_DIR = os.path.join(REPO, "baseline", "_ref")

# Qwen2-0.5B (the BASELINE config-5 model): 24 layers, hidden 896, 14 / 2
# heads of 64, SiLU-gated MLP 4864, vocab 151936, RoPE theta 1e6, RMSNorm 1e-6.
QWEN2_0_5B: Dict[str, Any] = {
    "model_type": "qwen2",
    "architectures": ["Qwen2ForCausalLM"],
    "num_hidden_layers": 24,
    "hidden_size": 896,
    "num_attention_heads": 14,
    "num_key_value_heads": 2,
    "intermediate_size": 4864,
    "vocab_size": 151936,
    "rms_norm_eps": 1e-6,
    "rope_theta": 1000000.0,
    "max_position_embeddings": 32768,
    "hidden_act": "silu",
    "tie_word_embeddings": True,
}


def import_reference():
    """Import the installed reference package ``mini_vllm`` (from
    ``baseline/_ref``); raises ImportError naming the install script when it
    is missing."""
    if REFERENCE_DIR not in sys.path and os.path.isdir(REFERENCE_DIR):
        sys.path.insert(0, REFERENCE_DIR)
    try:
        import mini_vllm  # noqa: F401
    except ImportError as e:  # pragma: no cover - depends on the install
        raise ImportError(
            f"the reference package mini_vllm is not installed in {REFERENCE_DIR}: "
            "run baseline/install_reference.sh") from e
    return sys.modules["mini_vllm"]


def register_backend(**backend_options) -> None:
    """Add the ``"b200"`` branch to the reference's ``AttentionBackend.create``
    (every other name keeps its original behaviour, including the
    ``ValueError`` for unknown names).  ``backend_options`` are passed to
    ``AttentionBackendB200`` (``strict``, ``overlap_after_write``, ...).
    Calling it again replaces the options."""
    import_reference()
    from mini_vllm.attention import backend as ref_backend

    cls = ref_backend.AttentionBackend
    original = getattr(cls, "_mvb_original_create", None)
    if original is None:
        original = cls.create
        cls._mvb_original_create = original

    def create(config, backend: str = "triton"):
        if backend == "b200":
            from .attention.paged_attention_b200 import AttentionBackendB200

            return AttentionBackendB200(config, **backend_options)
        return original(config, backend=backend)

    cls.create = staticmethod(create)


def write_random_checkpoint(path: str, *, num_layers: Optional[int] = None, vocab_size: Optional[int] = None,
                            seed: int = 0, std: float = 0.02, **overrides) -> Dict[str, Any]:
    """Write a random Qwen2 checkpoint directory at ``path`` and return its
    config.  Shapes default to Qwen2-0.5B; ``num_layers`` / ``vocab_size`` /
    other config keys override them (a test may use 2 layers).  Weights are
    drawn in float32 from a seeded generator on the CPU and stored as bf16."""
    import torch
    from safetensors.torch import save_file

    cfg = dict(QWEN2_0_5B)
    if num_layers is not None:
        cfg["num_hidden_layers"] = num_layers
    if vocab_size is not None:
        cfg["vocab_size"] = vocab_size
    cfg.update(overrides)
    os.makedirs(path, exist_ok=True)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f, indent=1)

    g = torch.Generator().manual_seed(seed)
    H, V, I = cfg["hidden_size"], cfg["vocab_size"], cfg["intermediate_size"]
    nh, nkv = cfg["num_attention_heads"], cfg["num_key_value_heads"]
    hd = cfg.get("head_dim", H // nh)

    def randn(*shape):
        return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)

    sd = {"model.embed_tokens.weight": randn(V, H), "model.norm.weight": torch.ones(H, dtype=torch.bfloat16)}
    if not cfg["tie_word_embeddings"]:
        sd["lm_head.weight"] = randn(V, H)
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}"
        sd[f"{p}.input_layernorm.weight"] = torch.ones(H, dtype=torch.bfloat16)
        sd[f"{p}.post_attention_layernorm.weight"] = torch.ones(H, dtype=torch.bfloat16)
        sd[f"{p}.self_attn.q_proj.weight"] = randn(nh * hd, H)
        sd[f"{p}.self_attn.q_proj.bias"] = randn(nh * hd)
        sd[f"{p}.self_attn.k_proj.weight"] = randn(nkv * hd, H)
        sd[f"{p}.self_attn.k_proj.bias"] = randn(nkv * hd)
        sd[f"{p}.self_attn.v_proj.weight"] = randn(nkv * hd, H)
        sd[f"{p}.self_attn.v_proj.bias"] = randn(nkv * hd)
        sd[f"{p}.self_attn.o_proj.weight"] = randn(H, nh * hd)
        sd[f"{p}.mlp.gate_proj.weight"] = randn(I, H)
        sd[f"{p}.mlp.up_proj.weight"] = randn(I, H)
        sd[f"{p}.mlp.down_proj.weight"] = randn(H, I)
    save_file(sd, os.path.join(path, "model.safetensors"))
    _write_id_tokenizer(path, V)
    return cfg


def _write_id_tokenizer(path: str, vocab_size: int) -> None:
    """A word-level tokenizer whose words are the decimal token ids, split on
    whitespace: what AutoTokenizer.from_pretrained loads for PagedExecutor."""
    from tokenizers import Tokenizer
    from tokenizers.models import WordLevel
    from tokenizers.pre_tokenizers import WhitespaceSplit
    from transformers import PreTrainedTokenizerFast

    # no special tokens: a special token's text is matched inside words ("0"
    # would split "300"), and prompts hold ids only, so nothing is unknown
    vocab = {str(i): i for i in range(vocab_size)}
    tok = Tokenizer(WordLevel(vocab, unk_token="<unk>"))
    tok.pre_tokenizer = WhitespaceSplit()
    PreTrainedTokenizerFast(tokenizer_object=tok).save_pretrained(path)


def prompt_text(token_ids) -> str:
    """The prompt string the id tokenizer encodes back to ``token_ids``."""
    return " ".join(str(int(t)) for t in token_ids)
