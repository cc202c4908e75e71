"""mini_vllm_b200 — B200-native paged-attention decode and KV-cache write for mini-vLLM.

A drop-in for the attention plug-in of lmjlmj1234/mini-vllm-continuous-batching-lab
(mini_vllm/attention): the same call signatures, backed by hand-written sm_100a
CUDA kernels in ``lib/libmvb200.so`` (sources in ``csrc/``, C ABI in
``include/mini_vllm_b200.h``).  Import it as ``mini_vllm_b200`` (the repository
root's ``mini_vllm_b200.py`` maps that name onto this directory).
"""

from .attention import (
    ArgumentError,
    AttentionBackend,
    AttentionBackendB200,
    DecodeSchedule,
    build_decode_schedule,
    check_device_errors,
    decode_plan,
    gather_paged_kv,
    gather_prefix_kv,
    paged_cache_write,
    paged_decode_attention,
    paged_gather,
    paged_prefill_attention,
    rope_cache_write,
    rope_tables,
    triton_cache_write,
    triton_decode_attention,
)
from .cache import KVCachePool, compute_num_gpu_blocks
from .engine import StepMetadata, StepMetadataBuilder
from .model_runner import AttentionGroup, AttentionMetadata, ModelConfig
from . import staging

__version__ = "0.1.0"

__all__ = [
    "staging",
    "ArgumentError",
    "AttentionBackend",
    "AttentionBackendB200",
    "DecodeSchedule",
    "build_decode_schedule",
    "AttentionGroup",
    "AttentionMetadata",
    "KVCachePool",
    "ModelConfig",
    "StepMetadata",
    "StepMetadataBuilder",
    "check_device_errors",
    "compute_num_gpu_blocks",
    "decode_plan",
    "gather_paged_kv",
    "gather_prefix_kv",
    "paged_cache_write",
    "paged_decode_attention",
    "paged_gather",
    "paged_prefill_attention",
    "rope_cache_write",
    "rope_tables",
    "triton_cache_write",
    "triton_decode_attention",
]
