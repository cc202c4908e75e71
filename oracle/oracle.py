"""Python side of the CPU oracle — TEST INFRASTRUCTURE ONLY.

Two restatements of the reference's CPU algorithm for the paged KV path:

* ``paged_oracle.c`` (built into ``liboracle.so`` by ``build_oracle``), C with
  OpenMP — fast enough to check BASELINE-size workloads and to serve as the
  timed CPU baseline;
* ``*_numpy`` functions below, plain numpy / Python loops for small cases, used
  to cross-check the C restatement.

Both are pinned to the reference by ``tests/golden`` (vectors produced by the
reference's own ``write_to_paged_cache`` and ``AttentionBackendRef``).

Arrays are numpy.  A bf16 tensor is passed as its raw ``uint16`` bits with
``dtype="bf16"``; ``"f16"`` arrays are ``float16``, ``"f32"`` arrays ``float32``.

Reference lines restated:
  cache_write  <- mini_vllm/cache/cache_write.py:25-74   (write_to_paged_cache)
  gather       <- mini_vllm/cache/cache_read.py:19-84     (gather_paged_kv)
  decode       <- mini_vllm/attention/paged_attention_ref.py:102-161
                  (AttentionBackendRef.decode_attention; torch SDPA math)
  rope_numpy   <- mini_vllm/model/rotary.py:47-85 (RotaryEmbedding.__call__,
                  _rotate_half), with the rounding of each torch operation
  step_metadata_numpy <- mini_vllm/engine/input_builder.py:48-256
                  (positions, _compute_slot, _build_block_table_tensor, sample indices)
"""

from __future__ import annotations

import ctypes
import os
import subprocess
import threading
from typing import Optional, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "paged_oracle.c")
LIB = os.path.join(HERE, "liboracle.so")

ORACLE_OK = 0
ORACLE_KV_LEN = 1
ORACLE_TABLE_SHORT = 2
ORACLE_BLOCK_ID = 3

_CODES = {"f32": 0, "f16": 1, "bf16": 2}
_lib = None
_lock = threading.Lock()


def build_oracle(force: bool = False) -> str:
    """Compile ``paged_oracle.c`` into ``liboracle.so`` with gcc + OpenMP."""
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < os.path.getmtime(SRC):
        cmd = ["gcc", "-O2", "-std=c11", "-fopenmp", "-fPIC", "-shared", SRC, "-o", LIB, "-lm"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"oracle build failed:\n{res.stderr}")
    return LIB


def _load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                build_oracle()
                h = ctypes.CDLL(LIB)
                vp, i64, i32, f64 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_double
                h.oracle_cache_write.restype = i32
                h.oracle_cache_write.argtypes = [vp, vp, vp, vp, vp, i64, i32, i32, i32, i64, i32]
                h.oracle_gather.restype = i32
                h.oracle_gather.argtypes = [vp, vp, vp, i64, i64, i32, i32, i32, i32, vp, vp]
                h.oracle_decode.restype = i32
                h.oracle_decode.argtypes = [vp, vp, vp, vp, i64, vp, i64, i32, i32, i32, i32, i64,
                                            f64, i32, i32, vp, vp]
                h.oracle_max_threads.restype = i32
                _lib = h
    return _lib


def max_threads() -> int:
    return int(_load().oracle_max_threads())


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def to_float32(a: np.ndarray, dtype: str) -> np.ndarray:
    """Upcast storage values to float32 (bf16 bits are widened by a 16-bit shift)."""
    if dtype == "bf16":
        return (a.astype(np.uint32) << 16).view(np.float32)
    return a.astype(np.float32)


def _c(a: np.ndarray, dt=None) -> np.ndarray:
    return np.ascontiguousarray(a if dt is None else a.astype(dt, copy=False))


# ---------------------------------------------------------------------------
# C restatement
# ---------------------------------------------------------------------------
def cache_write(key, value, key_cache, value_cache, slot_mapping, block_size: int, dtype: str) -> None:
    """In-place sequential scatter, last writer wins (cache_write.py:55-74).

    Raises IndexError for the first slot outside [0, num_blocks*block_size)
    other than -1, after writing the tokens before it, as the reference does.
    """
    assert key_cache.flags["C_CONTIGUOUS"] and value_cache.flags["C_CONTIGUOUS"]
    key, value = _c(key), _c(value)
    slots = _c(slot_mapping, np.int64)
    T, KH, D = key.shape
    NB = key_cache.shape[0]
    st = _load().oracle_cache_write(_ptr(key), _ptr(value), _ptr(key_cache), _ptr(value_cache),
                                    _ptr(slots), T, KH, D, block_size, NB, _CODES[dtype])
    if st < 0:
        t = -st - 1
        raise IndexError(
            f"slot_mapping[{t}] = {int(slots[t])} out of range [0, {NB * block_size}) "
            f"(block_size={block_size}, num_blocks={NB})"
        )


def gather(key_cache, value_cache, block_ids, num_tokens: int, block_size: int,
           dtype: str) -> Tuple[np.ndarray, np.ndarray]:
    """Contiguous [num_tokens, KH, D] K and V from the blocks in logical order."""
    NB, KH, BS, D = key_cache.shape
    ids = _c(np.asarray(block_ids, dtype=np.int64).reshape(-1))
    out_k = np.empty((num_tokens, KH, D), dtype=key_cache.dtype)
    out_v = np.empty((num_tokens, KH, D), dtype=key_cache.dtype)
    if num_tokens == 0:
        return out_k, out_v
    st = _load().oracle_gather(_ptr(_c(key_cache)), _ptr(_c(value_cache)), _ptr(ids), ids.size,
                               num_tokens, KH, D, block_size, _CODES[dtype], _ptr(out_k), _ptr(out_v))
    if st != 0:
        raise IndexError(
            f"block_table length {ids.size} insufficient to cover {num_tokens} tokens "
            f"(block_size={block_size})"
        )
    return out_k, out_v


def decode(query, key_cache, value_cache, block_table, kv_len, block_size: int, dtype: str,
           scale: Optional[float] = None, threads: int = 0) -> Tuple[np.ndarray, np.ndarray]:
    """Paged decode attention in float64 arithmetic; returns (out float32 [Nd,H,D], status [Nd])."""
    q = _c(query)
    Nd, H, D = q.shape
    NB, KH, BS, _ = key_cache.shape
    bt = _c(block_table, np.int64)
    if bt.ndim == 1:
        bt = bt.reshape(Nd, -1)
    kvl = _c(kv_len, np.int32)
    if scale is None:
        scale = D ** -0.5
    out = np.zeros((Nd, H, D), dtype=np.float32)
    status = np.zeros(Nd, dtype=np.int32)
    _load().oracle_decode(_ptr(q), _ptr(_c(key_cache)), _ptr(_c(value_cache)), _ptr(bt), bt.shape[1],
                          _ptr(kvl), Nd, H, KH, D, block_size, NB, float(scale), _CODES[dtype],
                          int(threads), _ptr(out), _ptr(status))
    return out, status


# ---------------------------------------------------------------------------
# numpy restatement (small cases)
# ---------------------------------------------------------------------------
def cache_write_numpy(key, value, key_cache, value_cache, slot_mapping, block_size: int) -> None:
    """Token loop of write_to_paged_cache (cache_write.py:55-74), on numpy arrays."""
    total = key_cache.shape[0] * block_size
    for t, slot in enumerate(np.asarray(slot_mapping).tolist()):
        if slot == -1:
            continue
        if slot < -1 or slot >= total:
            raise IndexError(f"slot_mapping[{t}] = {slot} out of range [0, {total})")
        key_cache[slot // block_size, :, slot % block_size, :] = key[t]
        value_cache[slot // block_size, :, slot % block_size, :] = value[t]


def decode_numpy(query, key_cache, value_cache, block_table, kv_len, block_size: int, dtype: str,
                 scale: Optional[float] = None) -> np.ndarray:
    """Per-sequence gather + repeat_interleave + softmax attention in float64
    (paged_attention_ref.py:132-161 with cache_read.py:40-84)."""
    q = to_float32(np.asarray(query), dtype).astype(np.float64)
    kc = to_float32(np.asarray(key_cache), dtype)
    vc = to_float32(np.asarray(value_cache), dtype)
    Nd, H, D = q.shape
    KH = kc.shape[1]
    G = H // KH
    if scale is None:
        scale = D ** -0.5
    out = np.zeros((Nd, H, D), dtype=np.float32)
    for s in range(Nd):
        n = int(kv_len[s])
        ids = [int(b) for b in np.asarray(block_table[s]).tolist() if b != -1]
        if (n + block_size - 1) // block_size > len(ids):
            raise IndexError(f"block_table length {len(ids)} insufficient to cover {n} tokens")
        pos = np.arange(n)
        blk = np.asarray(ids, dtype=np.int64)[pos // block_size]
        k = kc[blk, :, pos % block_size, :].astype(np.float64)  # [n, KH, D]
        v = vc[blk, :, pos % block_size, :].astype(np.float64)
        k = np.repeat(k, G, axis=1)  # repeat_interleave over heads
        v = np.repeat(v, G, axis=1)
        logits = np.einsum("hd,nhd->hn", q[s], k) * scale
        logits -= logits.max(axis=1, keepdims=True)
        p = np.exp(logits)
        p /= p.sum(axis=1, keepdims=True)
        out[s] = np.einsum("hn,nhd->hd", p, v).astype(np.float32)
    return out


# ---------------------------------------------------------------------------
# rotary embedding (numpy restatement)
# ---------------------------------------------------------------------------
def round_to_dtype(x32: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values rounded to `dtype` (round to nearest even), as float32."""
    x32 = np.asarray(x32, dtype=np.float32)
    if dtype == "f32":
        return x32
    if dtype == "f16":
        return x32.astype(np.float16).astype(np.float32)
    bits = x32.view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    nan = np.isnan(x32)
    out = (rounded.astype(np.uint32) << 16).view(np.float32).copy()
    out[nan] = x32[nan]
    return out


def from_float32(x32: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values already representable in `dtype` to the storage form."""
    if dtype == "bf16":
        return (np.asarray(x32, np.float32).view(np.uint32) >> 16).astype(np.uint16)
    return np.asarray(x32).astype(np.float16 if dtype == "f16" else np.float32)


def rope_numpy(x, positions, cos, sin, dtype: str) -> np.ndarray:
    """x * cos[pos] + rotate_half(x) * sin[pos] over [T, heads, D] (rotary.py:47-85).

    Each of the three torch operations rounds to the dtype: the products are
    formed in float32 (exact for 16-bit inputs) and rounded, their sum is a
    float32 add of the rounded products, rounded again."""
    xf = to_float32(np.asarray(x), dtype)
    pos = np.asarray(positions, dtype=np.int64)
    c = to_float32(np.asarray(cos), dtype)[pos][:, None, :]
    sn = to_float32(np.asarray(sin), dtype)[pos][:, None, :]
    half = xf.shape[-1] // 2
    rot = np.concatenate([-xf[..., half:], xf[..., :half]], axis=-1)
    a = round_to_dtype(xf * c, dtype)
    b = round_to_dtype(rot * sn, dtype)
    return from_float32(round_to_dtype(a + b, dtype), dtype)


# ---------------------------------------------------------------------------
# step metadata (numpy restatement)
# ---------------------------------------------------------------------------
def step_metadata_numpy(block_lists, cached, query_len, completes, num_prefill: int, block_size: int):
    """positions, slot_mapping, prefill / decode block tables (-1 padded to the
    step's longest table, at least 1; (0, 0) for an empty phase), sample token
    indices and kv_len_after of one step, sequences prefill first
    (input_builder.py:48-256).  Raises RuntimeError("Block not allocated ...")
    for a position past a sequence's blocks, as _compute_slot does."""
    S = len(block_lists)
    positions, slots, sample = [], [], []
    tok = 0
    for s in range(S):
        blocks = list(block_lists[s])
        for i in range(int(query_len[s])):
            pos = int(cached[s]) + i
            lb = pos // block_size
            if lb >= len(blocks):
                raise RuntimeError(f"Block not allocated for position={pos} (logical_idx={lb}, "
                                   f"num_blocks={len(blocks)})")
            positions.append(pos)
            slots.append(blocks[lb] * block_size + pos % block_size)
        if s < num_prefill:
            if completes[s]:
                sample.append(tok + int(query_len[s]) - 1)
        else:
            sample.append(tok)
        tok += int(query_len[s])
    max_blocks = max(1, max((len(b) for b in block_lists), default=0))

    def table(rows):
        if not rows:
            return np.zeros((0, 0), dtype=np.int64)
        return np.array([list(b) + [-1] * (max_blocks - len(b)) for b in rows], dtype=np.int64)

    kv_len = np.array([int(c) + int(q) for c, q in zip(cached, query_len)], dtype=np.int64)
    return (np.array(positions, dtype=np.int64), np.array(slots, dtype=np.int64),
            table(block_lists[:num_prefill]), table(block_lists[num_prefill:]),
            np.array(sample, dtype=np.int64), kv_len)
