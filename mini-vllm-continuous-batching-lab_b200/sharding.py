"""Sequence sharding of a paged decode across GPUs, and the output gather.

Sequences are independent in decode attention and each owns its KV blocks, so
the batch is partitioned by sequence with no exchange inside attention: every
rank holds its own KV pool and block tables and runs the kernels on its share.
The only collective is one all-gather of the per-rank outputs (NCCL over
NVLink when the group is NCCL; gloo on CPU in the tests), after which rank 0
(or every rank) reorders rows back to the global sequence order.

Assignment is token-balanced with equal sequence counts: sequences sorted by
context length (longest first) are dealt to ranks in snake order
0,1,..,R-1,R-1,..,0,0,1,... so each rank's token total is close to B*mean/R.
"""

from __future__ import annotations

from typing import List

import numpy as np


def snake_assignment(context_lens: np.ndarray, world_size: int) -> List[np.ndarray]:
    """Global sequence indices owned by each rank (each list sorted ascending)."""
    ctx = np.asarray(context_lens, dtype=np.int64)
    if world_size < 1:
        raise ValueError(f"world_size must be >= 1, got {world_size}")
    order = np.argsort(-ctx, kind="stable")
    owners: List[List[int]] = [[] for _ in range(world_size)]
    for pos, seq in enumerate(order.tolist()):
        rnd, k = divmod(pos, world_size)
        rank = k if rnd % 2 == 0 else world_size - 1 - k
        owners[rank].append(seq)
    return [np.sort(np.asarray(o, dtype=np.int64)) for o in owners]


class OutputGather:
    """Reusable all-gather of per-rank ``[n_rank, H, D]`` outputs into global order.

    The buffers and the permutation are built once on the device, so one call
    is a single ``all_gather_into_tensor`` plus one ``index_select`` into the
    output (global row g <- received row ``perm[g]``) — no host work, no
    allocation, capturable in a CUDA graph.  A decode that writes its output
    into ``send_view(n)`` (``decode_attention(out=...)``) saves the copy into
    the send buffer.
    """

    def __init__(self, owned: List[np.ndarray], heads: int, head_dim: int, dtype, device, group=None):
        import torch

        self.world = len(owned)
        self.counts = [int(o.size) for o in owned]
        self.cap = max(self.counts) if self.counts else 0
        self.group = group
        self.total = sum(self.counts)
        self.send = torch.zeros((self.cap, heads, head_dim), dtype=dtype, device=device)
        self.recv = torch.empty((self.world * self.cap, heads, head_dim), dtype=dtype, device=device)
        self.out = torch.empty((self.total, heads, head_dim), dtype=dtype, device=device)
        # received row of every global sequence (rank r's i-th owned sequence
        # arrives at row r * cap + i)
        perm = np.zeros(self.total, np.int64)
        for r, o in enumerate(owned):
            perm[np.asarray(o, dtype=np.int64)] = r * self.cap + np.arange(o.size)
        self.perm = torch.from_numpy(perm).to(device)

    def send_view(self, n: int):
        """The first ``n`` rows of the send buffer: a decode's ``out=`` target."""
        return self.send[:n]

    def __call__(self, local_out):
        import torch
        import torch.distributed as dist

        n = local_out.shape[0]
        if local_out.data_ptr() != self.send.data_ptr():
            self.send[:n].copy_(local_out)
        dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        torch.index_select(self.recv, 0, self.perm, out=self.out)
        return self.out


def gather_outputs(local_out, owned: List[np.ndarray], rank: int, group=None):
    """All-gather every rank's ``local_out`` ([n_rank, H, D]) and return the
    ``[B, H, D]`` result in global sequence order (on every rank).

    Ranks with fewer sequences pad to the largest share so one
    ``all_gather_into_tensor`` moves everything; the padding is dropped when
    the rows are scattered back into global order.
    """
    import torch
    import torch.distributed as dist

    world = len(owned)
    counts = [int(o.size) for o in owned]
    cap = max(counts) if counts else 0
    h, d = local_out.shape[1], local_out.shape[2]
    send = local_out
    if local_out.shape[0] < cap:
        send = torch.zeros((cap, h, d), dtype=local_out.dtype, device=local_out.device)
        send[: local_out.shape[0]] = local_out
    recv = torch.empty((world * cap, h, d), dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(recv, send.contiguous(), group=group)
    total = sum(counts)
    out = torch.empty((total, h, d), dtype=local_out.dtype, device=local_out.device)
    for r in range(world):
        if counts[r]:
            idx = torch.from_numpy(owned[r]).to(local_out.device)
            out[idx] = recv[r * cap: r * cap + counts[r]]
    return out
