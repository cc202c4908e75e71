"""The attention plug-in interface (mirror of mini_vllm/attention/backend.py:12-113).

``AttentionBackend`` keeps the reference's four methods with the same
arguments, so the reference's model runner (qwen_runner.py:168-190) drives the
B200 backend unchanged:

* ``allocate_pool`` (reference :27-44) — allocate the per-layer K/V pool;
* ``write_kv_cache`` (reference :46-61) — scatter new K/V rows by slot;
* ``decode_attention`` (reference :63-77) — paged decode, one query per sequence;
* ``prefill_attention`` (reference :79-96) — prefill over the paged prefix.

``create`` only knows the B200 backend: there is no multi-backend dispatch and
no silent fallback, an unknown name raises ``ValueError`` (reference :112-113).
"""

from __future__ import annotations

from abc import ABC, abstractmethod
from typing import Any

import torch


class AttentionBackend(ABC):
    @abstractmethod
    def allocate_pool(
        self,
        num_layers: int,
        num_blocks: int,
        block_size: int,
        num_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype,
        device: torch.device,
    ) -> Any:
        """Allocate the KV pool; returns an object with ``key_caches`` / ``value_caches``."""

    @abstractmethod
    def write_kv_cache(
        self,
        layer_idx: int,
        key: torch.Tensor,  # [num_tokens, num_kv_heads, head_dim]
        value: torch.Tensor,  # [num_tokens, num_kv_heads, head_dim]
        slot_mapping: torch.Tensor,  # [num_tokens] int64, -1 = skip
    ) -> None:
        """Scatter-write K/V rows into layer ``layer_idx`` of the pool."""

    @abstractmethod
    def decode_attention(
        self,
        layer_idx: int,
        query: torch.Tensor,  # [num_decode_tokens, num_heads, head_dim]
        attn_metadata: Any,
        pool: Any,
    ) -> torch.Tensor:
        """Paged decode attention over each sequence's own blocks."""

    @abstractmethod
    def prefill_attention(
        self,
        layer_idx: int,
        query: torch.Tensor,
        key: torch.Tensor,
        value: torch.Tensor,
        attn_metadata: Any,
        pool: Any,
    ) -> torch.Tensor:
        """Causal prefill attention over the cached prefix plus the chunk."""

    @staticmethod
    def create(config: Any, backend: str = "b200", **kwargs: Any) -> "AttentionBackend":
        """Factory.  ``backend`` must be ``"b200"`` (alias ``"cuda"``)."""
        if backend in ("b200", "cuda"):
            from .paged_attention_b200 import AttentionBackendB200

            return AttentionBackendB200(config, **kwargs)
        raise ValueError(f"Unknown AttentionBackend: {backend!r}")
