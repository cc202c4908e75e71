"""Seeded synthetic paged-decode workloads with the shapes of the benchmark configs.

No dataset is involved anywhere on this path: every config is synthetic.  The
block-table construction mirrors what the reference's input builder produces
(int64 rows, ``-1`` padded to the batch's widest row; input_builder.py:239-258):
each sequence owns ``ceil(ctx / block_size)`` physical blocks drawn without
overlap from a seeded permutation of the pool.

Configs (numbered as in the benchmark plan):

1. CPU-size check: batch 8, ctx ~ U{1..512}, 14 q / 2 KV heads, head_dim 64,
   block 16, a fixed pool of 512 blocks, fp32.
2. 1-GPU headline: batch 256, ctx ~ U{128..2048}, 14/2/64, block 16, pool =
   ceil(1.1 * blocks needed), bf16.
3. long context: batch 32, ctx = 32768 each, 14/2/64, block 16, split-K.
4. larger GQA, sharded across GPUs: 32/8/128, global batch 1024,
   ctx = clip(round(lognormal(7.0, 0.8)), 16, 8192), block 16.

Every config also carries the decode step's KV write: one new token per
sequence at position ``ctx - 1`` (write-first: ``kv_len_after = ctx``), i.e.
``slot = table[s][(ctx-1) // BS] * BS + (ctx-1) % BS``.

Tensor contents (q, K, V ~ N(0, 1)) are produced by ``numpy_tensors`` (CPU,
deterministic across machines) or ``torch_tensors`` (on the device, fast).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import numpy as np


@dataclass
class PagedDecodeSpec:
    name: str
    num_seqs: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    block_size: int
    num_blocks: int
    context_lens: np.ndarray  # int64 [B]
    block_tables: np.ndarray  # int64 [B, max_blocks], -1 padded
    slot_mapping: np.ndarray  # int64 [B], the new token of each sequence
    seed: int

    @property
    def max_blocks(self) -> int:
        return int(self.block_tables.shape[1])

    @property
    def total_tokens(self) -> int:
        return int(self.context_lens.sum())

    def kv_bytes(self, esize: int) -> int:
        """K+V bytes one decode reads (each KV head's tokens once)."""
        return self.total_tokens * 2 * self.num_kv_heads * self.head_dim * esize

    def decode_bytes(self, esize: int) -> int:
        """Algorithmic HBM bytes of one decode call.

        K+V once per KV head, the query read and the output written, the
        block-table entries actually read (8 bytes each) and the int32 context
        lengths.
        """
        blocks_read = int(((self.context_lens + self.block_size - 1) // self.block_size).sum())
        return (self.kv_bytes(esize)
                + 2 * self.num_seqs * self.num_heads * self.head_dim * esize
                + 8 * blocks_read + 4 * self.num_seqs)

    def write_bytes(self, esize: int) -> int:
        """Algorithmic bytes of the step's KV write: rows read + written, slots read."""
        return 2 * 2 * self.num_seqs * self.num_kv_heads * self.head_dim * esize + 8 * self.num_seqs

    def decode_flops(self) -> int:
        return 4 * self.total_tokens * self.num_heads * self.head_dim


CONFIGS: Dict[int, Dict] = {
    1: dict(num_seqs=8, num_heads=14, num_kv_heads=2, head_dim=64, block_size=16, ctx=("uniform", 1, 512),
            num_blocks=512),
    2: dict(num_seqs=256, num_heads=14, num_kv_heads=2, head_dim=64, block_size=16,
            ctx=("uniform", 128, 2048), num_blocks=None),
    3: dict(num_seqs=32, num_heads=14, num_kv_heads=2, head_dim=64, block_size=16,
            ctx=("const", 32768, 32768), num_blocks=None),
    4: dict(num_seqs=1024, num_heads=32, num_kv_heads=8, head_dim=128, block_size=16,
            ctx=("lognormal", 7.0, 0.8), num_blocks=None),
}


def context_lengths(config: int, seed: int = 0, num_seqs: Optional[int] = None) -> np.ndarray:
    c = CONFIGS[config]
    n = c["num_seqs"] if num_seqs is None else num_seqs
    rng = np.random.default_rng(seed)
    kind, a, b = c["ctx"]
    if kind == "uniform":
        return rng.integers(a, b + 1, size=n).astype(np.int64)
    if kind == "const":
        return np.full(n, a, dtype=np.int64)
    ctx = np.rint(rng.lognormal(mean=a, sigma=b, size=n))
    return np.clip(ctx, 16, 8192).astype(np.int64)


def build_spec(name: str, context_lens: np.ndarray, num_heads: int, num_kv_heads: int, head_dim: int,
               block_size: int, num_blocks: Optional[int] = None, seed: int = 0) -> PagedDecodeSpec:
    """Block tables and write slots for the given context lengths."""
    ctx = np.asarray(context_lens, dtype=np.int64)
    nblk = (ctx + block_size - 1) // block_size
    need = int(nblk.sum())
    if num_blocks is None:
        num_blocks = max(16, int(np.ceil(1.1 * need)))
    if need > num_blocks:
        raise ValueError(f"pool of {num_blocks} blocks cannot hold {need} blocks")
    rng = np.random.default_rng(seed + 7919)
    perm = rng.permutation(num_blocks).astype(np.int64)
    width = int(nblk.max()) if ctx.size else 1
    tables = np.full((ctx.size, width), -1, dtype=np.int64)
    off = 0
    for i, k in enumerate(nblk.tolist()):
        tables[i, :k] = perm[off:off + k]
        off += k
    last = ctx - 1
    slots = (tables[np.arange(ctx.size), last // block_size] * block_size + last % block_size
             if ctx.size else np.zeros(0, dtype=np.int64))
    return PagedDecodeSpec(name, int(ctx.size), num_heads, num_kv_heads, head_dim, block_size,
                           int(num_blocks), ctx, tables, slots.astype(np.int64), seed)


def make_spec(config: int, seed: int = 0, num_seqs: Optional[int] = None) -> PagedDecodeSpec:
    c = CONFIGS[config]
    ctx = context_lengths(config, seed, num_seqs)
    return build_spec(f"config{config}", ctx, c["num_heads"], c["num_kv_heads"], c["head_dim"],
                      c["block_size"], c["num_blocks"], seed)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16, returned as uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    return (rounded >> np.uint32(16)).astype(np.uint16)


def numpy_tensors(spec: PagedDecodeSpec, dtype: str, seed: Optional[int] = None) -> Dict[str, np.ndarray]:
    """q [B,H,D], key/value caches [NB,KH,BS,D], new_key/new_value [B,KH,D] ~ N(0,1).

    ``dtype`` is "f32", "f16" or "bf16" (bf16 returned as uint16 bits).
    """
    rng = np.random.default_rng(spec.seed + 104729 if seed is None else seed)
    shapes = {
        "query": (spec.num_seqs, spec.num_heads, spec.head_dim),
        "key_cache": (spec.num_blocks, spec.num_kv_heads, spec.block_size, spec.head_dim),
        "value_cache": (spec.num_blocks, spec.num_kv_heads, spec.block_size, spec.head_dim),
        "new_key": (spec.num_seqs, spec.num_kv_heads, spec.head_dim),
        "new_value": (spec.num_seqs, spec.num_kv_heads, spec.head_dim),
    }
    out = {}
    for k, shp in shapes.items():
        x = rng.standard_normal(shp, dtype=np.float32)
        if dtype == "bf16":
            out[k] = f32_to_bf16_bits(x)
        elif dtype == "f16":
            out[k] = x.astype(np.float16)
        else:
            out[k] = x
    return out


def torch_tensors(spec: PagedDecodeSpec, dtype, device, seed: Optional[int] = None, num_layers: int = 1):
    """Device tensors for ``spec``: dict with query, new_key, new_value and
    per-layer lists key_caches / value_caches, plus block_tables, kv_len
    (int32) and slot_mapping on the device."""
    import torch

    g = torch.Generator(device=device)
    g.manual_seed(spec.seed + 104729 if seed is None else seed)

    def randn(*shape):
        return torch.randn(*shape, generator=g, device=device, dtype=torch.float32).to(dtype)

    cache_shape = (spec.num_blocks, spec.num_kv_heads, spec.block_size, spec.head_dim)
    return {
        "query": randn(spec.num_seqs, spec.num_heads, spec.head_dim),
        "new_key": randn(spec.num_seqs, spec.num_kv_heads, spec.head_dim),
        "new_value": randn(spec.num_seqs, spec.num_kv_heads, spec.head_dim),
        "key_caches": [randn(*cache_shape) for _ in range(num_layers)],
        "value_caches": [randn(*cache_shape) for _ in range(num_layers)],
        "block_tables": torch.from_numpy(spec.block_tables).to(device),
        "kv_len": torch.from_numpy(spec.context_lens.astype(np.int32)).to(device),
        "slot_mapping": torch.from_numpy(spec.slot_mapping).to(device),
    }
