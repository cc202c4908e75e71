"""Physical KV pool: the HBM layout the B200 kernels read and write.

Same contract as the reference's ``KVCachePool`` (mini_vllm/cache/pool.py:37-166):
one key and one value tensor per layer, each

    [num_blocks, num_kv_heads, block_size, head_dim]   contiguous, torch.empty

so a physical block id indexes dimension 0 of every layer.  In HBM one
(block, KV head) pair is a contiguous ``block_size * head_dim`` run — 2 KiB for
bf16 at block_size 16 / head_dim 64 — which is the unit the decode kernel's
TMA tile loads move (16 token rows at a time).  Memory is not zeroed: readers
never look past ``kv_len`` (the decode kernel masks and zeroes the tail of a
partial last tile in shared memory instead).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional

import torch

# Fewest blocks any pool may have (reference pool.py:26).
MIN_BLOCKS = 16
# Reserve for kernel workspaces when budgeting from free memory (reference pool.py:29).
_WORKSPACE_RESERVE = 256 * 1024 * 1024


@dataclass
class KVCachePool:
    key_caches: List[torch.Tensor]
    value_caches: List[torch.Tensor]
    num_blocks: int
    block_size: int
    num_layers: int
    num_kv_heads: int
    head_dim: int
    device: torch.device
    dtype: torch.dtype

    @staticmethod
    def allocate(
        num_layers: int,
        num_blocks: int,
        block_size: int,
        num_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype = torch.float16,
        device: Optional[torch.device] = None,
    ) -> "KVCachePool":
        """Allocate one uninitialised (K, V) tensor pair per layer.

        Raises ValueError for a non-positive dimension (reference pool.py:80-89).
        """
        for name, v in (
            ("num_blocks", num_blocks),
            ("num_layers", num_layers),
            ("block_size", block_size),
            ("num_kv_heads", num_kv_heads),
            ("head_dim", head_dim),
        ):
            if v <= 0:
                raise ValueError(f"{name} must be > 0, got {v}")
        dev = (
            torch.device(device)
            if device is not None
            else torch.device("cuda" if torch.cuda.is_available() else "cpu")
        )
        shape = (num_blocks, num_kv_heads, block_size, head_dim)
        keys = [torch.empty(shape, dtype=dtype, device=dev) for _ in range(num_layers)]
        values = [torch.empty(shape, dtype=dtype, device=dev) for _ in range(num_layers)]
        return KVCachePool(keys, values, num_blocks, block_size, num_layers, num_kv_heads,
                           head_dim, dev, dtype)

    def get_key_cache(self, layer_idx: int) -> torch.Tensor:
        return self.key_caches[layer_idx]

    def get_value_cache(self, layer_idx: int) -> torch.Tensor:
        return self.value_caches[layer_idx]

    def reset(self) -> None:
        """Zero every cache tensor."""
        for k, v in zip(self.key_caches, self.value_caches):
            k.zero_()
            v.zero_()

    @property
    def total_slots(self) -> int:
        """Token slots of one layer."""
        return self.num_blocks * self.block_size

    @property
    def bytes_per_block_per_layer(self) -> int:
        return 2 * self.num_kv_heads * self.block_size * self.head_dim * self.dtype.itemsize

    @property
    def bytes_per_block_total(self) -> int:
        return self.num_layers * self.bytes_per_block_per_layer

    @property
    def total_bytes(self) -> int:
        return self.num_blocks * self.bytes_per_block_total


def compute_num_gpu_blocks(
    num_layers: int,
    num_kv_heads: int,
    head_dim: int,
    block_size: int,
    dtype: torch.dtype = torch.float16,
    device: Optional[torch.device] = None,
    gpu_memory_utilization: float = 0.90,
    peak_runtime_estimate: int = 0,
    workspace_reserve: int = _WORKSPACE_RESERVE,
    num_gpu_blocks_override: Optional[int] = None,
) -> int:
    """Blocks that fit in free device memory (budget rule of reference pool.py:174-278).

    ``budget = (free - peak_runtime_estimate - workspace_reserve) * utilization``
    divided by the bytes one block takes across all layers (K and V), never
    below ``MIN_BLOCKS``.  An override is returned as-is after the minimum check.
    """
    if not (0 < gpu_memory_utilization <= 1.0):
        raise ValueError(f"gpu_memory_utilization must be in (0, 1], got {gpu_memory_utilization}")
    if num_gpu_blocks_override is not None:
        if num_gpu_blocks_override < MIN_BLOCKS:
            raise RuntimeError(
                f"num_gpu_blocks_override ({num_gpu_blocks_override}) < minimum ({MIN_BLOCKS})"
            )
        return num_gpu_blocks_override
    dev = (
        torch.device(device)
        if device is not None
        else torch.device("cuda" if torch.cuda.is_available() else "cpu")
    )
    if dev.type != "cuda":
        return MIN_BLOCKS
    free_bytes, _ = torch.cuda.mem_get_info(dev)
    post = free_bytes - peak_runtime_estimate - workspace_reserve
    if post <= 0:
        raise RuntimeError(
            f"GPU memory exhausted after deductions: free={free_bytes}, "
            f"peak={peak_runtime_estimate}, workspace={workspace_reserve}"
        )
    budget = int(post * gpu_memory_utilization)
    per_block = num_layers * 2 * num_kv_heads * block_size * head_dim * dtype.itemsize
    return max(MIN_BLOCKS, budget // per_block)
