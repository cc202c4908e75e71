from .backend import AttentionBackend
from .paged_attention_b200 import (
    ArgumentError,
    AttentionBackendB200,
    check_device_errors,
    decode_plan,
    gather_paged_kv,
    gather_prefix_kv,
    paged_cache_write,
    paged_decode_attention,
    paged_gather,
    triton_cache_write,
    triton_decode_attention,
    validate_block_size,
)

__all__ = [
    "ArgumentError",
    "AttentionBackend",
    "AttentionBackendB200",
    "check_device_errors",
    "decode_plan",
    "gather_paged_kv",
    "gather_prefix_kv",
    "paged_cache_write",
    "paged_decode_attention",
    "paged_gather",
    "triton_cache_write",
    "triton_decode_attention",
    "validate_block_size",
]
