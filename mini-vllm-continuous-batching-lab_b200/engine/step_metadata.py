"""Per-step attention metadata built on the device.

The tensors the attention path consumes each engine step — positions, slot
mapping, ``-1``-padded block tables and ``kv_len_after`` — with the values of
``ModelInputBuilder.build`` (mini_vllm/engine/input_builder.py:48-196), whose
per-token Python loops (``_compute_slot``, :202-221) and row padding
(``_build_block_table_tensor``, :238-256) dominate the host side of a step at
batch 256.  Here the host packs the step's block lists and lengths into one
pinned buffer, makes one copy, and ``mvb_build_step_metadata`` fills every
output in one launch.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import numpy as np
import torch

from .. import _native
from ..attention.paged_attention_b200 import _host_status, _state, _stream_handle, _take_flags


@dataclass
class StepMetadata:
    """Outputs of one step (device tensors; prefill tokens / rows first)."""
    positions: torch.Tensor             # int64 [T]
    slot_mapping: torch.Tensor          # int64 [T]
    prefill_block_tables: torch.Tensor  # int64 [P, max_blocks] (-1 padded), (0, 0) without prefill
    decode_block_tables: torch.Tensor   # int64 [D, max_blocks] (-1 padded), (0, 0) without decodes
    kv_len_after: torch.Tensor          # int32 [P + D]
    sample_token_indices: torch.Tensor  # int64: last token of completed prefills, every decode token
    num_prefill_tokens: int

    @property
    def decode_kv_len_after(self) -> torch.Tensor:
        """``kv_len_after`` of the decode sequences (the decode kernel's input)."""
        return self.kv_len_after[self.kv_len_after.shape[0] - self.decode_block_tables.shape[0]:]

    @property
    def prefill_slot_mapping(self) -> torch.Tensor:
        return self.slot_mapping[:self.num_prefill_tokens]

    @property
    def decode_slot_mapping(self) -> torch.Tensor:
        return self.slot_mapping[self.num_prefill_tokens:]


class StepMetadataBuilder:
    """Builds :class:`StepMetadata` for one engine step.

    ``prefill``: one ``(block_ids, cached_len_before, query_len, completes)``
    per prefill sequence; ``decode``: one ``(block_ids, cached_len_before)``
    per decode sequence (query length 1).  ``block_ids`` is the sequence's
    block table in logical order (``BlockManager.get_block_table``).  A token
    whose position has no block raises ``RuntimeError`` ("Block not
    allocated", input_builder.py:214-219).
    """

    def __init__(self, block_size: int, device: torch.device) -> None:
        if block_size <= 0:
            raise ValueError(f"block_size must be > 0, got {block_size}")
        self.block_size = block_size
        self.device = torch.device(device)

    @staticmethod
    def _staging(n: int) -> torch.Tensor:
        # A fresh pinned buffer per step from torch's caching host allocator,
        # which reuses a block only after the copies reading it have finished
        # (a buffer kept across steps could be overwritten under a pending copy).
        return torch.empty(n, dtype=torch.int64, pin_memory=True)

    def build(self, prefill: Sequence[Tuple[Sequence[int], int, int, bool]],
              decode: Sequence[Tuple[Sequence[int], int]], *, strict: bool = True) -> StepMetadata:
        """One step from per-sequence block lists (the reference builder's inputs)."""
        P, D = len(prefill), len(decode)
        lists = [np.asarray(p[0], dtype=np.int64).reshape(-1) for p in prefill] + \
                [np.asarray(d[0], dtype=np.int64).reshape(-1) for d in decode]
        counts = np.array([x.size for x in lists], dtype=np.int64)
        starts = np.zeros(P + D, dtype=np.int64)
        if P + D > 1:
            np.cumsum(counts[:-1], out=starts[1:])
        blocks = np.concatenate(lists) if lists else np.zeros(0, dtype=np.int64)
        cached = np.array([int(p[1]) for p in prefill] + [int(d[1]) for d in decode], dtype=np.int64)
        qlen = np.array([int(p[2]) for p in prefill] + [1] * D, dtype=np.int64)
        return self._launch(blocks, starts, counts, cached, qlen, [bool(p[3]) for p in prefill], P, strict)

    def build_from_arrays(self, tables: np.ndarray, counts: np.ndarray, cached: np.ndarray,
                          query_len: np.ndarray, completes: Sequence[bool], num_prefill: int, *,
                          strict: bool = True) -> StepMetadata:
        """One step from a padded ``[S, W]`` int64 table whose row s holds
        sequence s's block ids in its first ``counts[s]`` entries (prefill
        rows first), the form an engine keeps its tables in: no per-list
        conversion, one packed copy."""
        tables = np.ascontiguousarray(tables, dtype=np.int64)
        S = tables.shape[0]
        counts = np.asarray(counts, dtype=np.int64)
        if counts.shape != (S,) or (S and counts.max(initial=0) > tables.shape[1]):
            raise ValueError("counts must give one length <= the table width per row")
        starts = np.arange(S, dtype=np.int64) * (tables.shape[1] if tables.ndim == 2 else 0)
        return self._launch(tables.reshape(-1), starts, counts, np.asarray(cached, dtype=np.int64),
                            np.asarray(query_len, dtype=np.int64), list(completes), num_prefill, strict)

    def _launch(self, blocks, starts, counts, cached, qlen, completes, P: int, strict: bool) -> StepMetadata:
        S = starts.shape[0]
        D = S - P
        tok_off = np.zeros(S + 1, dtype=np.int64)
        if S:
            np.cumsum(qlen, out=tok_off[1:])
        T = int(tok_off[-1])
        max_blocks = max(1, int(counts.max(initial=0)))
        dev = self.device
        # sample indices (host: they only depend on the lengths and completion flags)
        done = np.asarray(completes, dtype=bool)
        sample = np.concatenate([(tok_off[:P] + qlen[:P] - 1)[done], tok_off[P:S]]).astype(np.int64)
        ns, nb = sample.size, blocks.size
        # one packed upload: starts, counts, token offsets, cached lengths, sample indices, block ids
        host = self._staging(4 * S + 1 + ns + nb)
        h = host.numpy()
        h[:S] = starts
        h[S:2 * S] = counts
        h[2 * S:3 * S + 1] = tok_off
        h[3 * S + 1:4 * S + 1] = cached
        h[4 * S + 1:4 * S + 1 + ns] = sample
        h[4 * S + 1 + ns:] = blocks
        buf = host.to(dev, non_blocking=True)
        positions = torch.empty(T, dtype=torch.int64, device=dev)
        slots = torch.empty(T, dtype=torch.int64, device=dev)
        tables = torch.empty((S, max_blocks), dtype=torch.int64, device=dev)
        kv_len = torch.empty(S, dtype=torch.int32, device=dev)
        sample_t = buf[4 * S + 1:4 * S + 1 + ns]
        if S:
            idx = dev.index if dev.index is not None else torch.cuda.current_device()
            state = _state(idx)
            base = buf.data_ptr()
            status = _native.lib().mvb_build_step_metadata(
                base + 8 * (4 * S + 1 + ns), base, base + 8 * S, base + 8 * (3 * S + 1), base + 8 * 2 * S,
                S, T, max_blocks, self.block_size, positions.data_ptr(), slots.data_ptr(), tables.data_ptr(),
                kv_len.data_ptr(), state.err_ptr, _stream_handle(idx))
            _host_status(status, "step metadata")
            if strict:
                flags = _take_flags(state)
                if flags & _native.DEV_TABLE_SHORT:
                    raise RuntimeError("Block not allocated for a token position of this step "
                                       "(its logical block is past the sequence's block table)")
        empty = torch.zeros((0, 0), dtype=torch.int64, device=dev)
        return StepMetadata(positions=positions, slot_mapping=slots,
                            prefill_block_tables=tables[:P] if P else empty,
                            decode_block_tables=tables[P:] if D else empty,
                            kv_len_after=kv_len, sample_token_indices=sample_t,
                            num_prefill_tokens=int(tok_off[P]))
