"""Per-step metadata types the attention plug-in reads.

Field-for-field mirrors of the reference's carriers
(mini_vllm/model_runner/base.py:14-84) so the B200 backend accepts either
these or the reference's own objects (it only reads attributes).

* ``AttentionGroup`` (reference :47-59): one attention type's sequences with
  ``cached_len_before``, ``query_len`` and ``kv_len_after`` (int64 tensors).
* ``AttentionMetadata`` (reference :62-84): the groups plus int64 ``-1``-padded
  block tables and slot mappings for the prefill and decode slices.
* ``ModelConfig`` (reference :14-40): model dimensions; the backend reads
  ``head_dim`` (and ``num_kv_heads``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch


def _empty_long() -> torch.Tensor:
    return torch.tensor([], dtype=torch.long)


@dataclass
class ModelConfig:
    model_type: str = ""
    num_layers: int = 0
    hidden_size: int = 0
    num_heads: int = 0
    num_kv_heads: int = 0
    head_dim: int = 0
    vocab_size: int = 0
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    max_position_embeddings: int = 32768
    hidden_act: str = "silu"
    intermediate_size: int = 0
    tie_word_embeddings: bool = True
    rope_scaling: Optional[dict] = None
    dtype: torch.dtype = torch.float16
    activation_dtype: torch.dtype = torch.float16


@dataclass
class AttentionGroup:
    seq_indices: List[int]
    attention_type: str  # "prefill_ref" | "prefill_gpu" | "decode_gpu"
    cached_len_before: torch.Tensor
    query_len: torch.Tensor
    kv_len_after: torch.Tensor


@dataclass
class AttentionMetadata:
    groups: List[AttentionGroup] = field(default_factory=list)
    prefill_slot_mapping: torch.Tensor = field(default_factory=_empty_long)
    prefill_block_tables: torch.Tensor = field(default_factory=_empty_long)
    prefill_positions: torch.Tensor = field(default_factory=_empty_long)
    decode_block_tables: torch.Tensor = field(default_factory=_empty_long)
    decode_slot_mapping: torch.Tensor = field(default_factory=_empty_long)
    decode_positions: torch.Tensor = field(default_factory=_empty_long)
    block_size: int = 0
    num_kv_heads: int = 0
    head_dim: int = 0
