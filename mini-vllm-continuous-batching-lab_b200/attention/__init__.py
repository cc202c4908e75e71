from .backend import AttentionBackend
from .paged_attention_b200 import (
    ArgumentError,
    AttentionBackendB200,
    check_device_errors,
    decode_plan,
    paged_cache_write,
    paged_decode_attention,
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
    "paged_cache_write",
    "paged_decode_attention",
    "triton_cache_write",
    "triton_decode_attention",
    "validate_block_size",
]
