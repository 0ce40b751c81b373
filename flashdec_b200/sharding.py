"""Request sharding of a ragged decode batch across the GPUs of one node.

Decode attention of one request touches only that request's KV pages, so a
batch shards by request with no collective on the data path: each rank owns
its requests' paged KV blocks and block tables.  The only optional exchange is
gathering per-step outputs back to the caller's rank (NCCL all-gather of the
padded ``[B_r, Hq, D]`` outputs over NVLink).

``lpt_partition`` is the longest-processing-time-first heuristic: requests in
decreasing length order, each to the rank with the least total length so far
(ties to the lower rank).  Its makespan is within 4/3 of optimal.
"""

from __future__ import annotations

import heapq
from typing import Sequence


def lpt_partition(lengths: Sequence[int], num_ranks: int) -> list[list[int]]:
    """Assign request indices to ``num_ranks`` shards balancing total length.

    Deterministic: requests are taken by decreasing length (then index) and
    each goes to the currently lightest rank (then lowest rank id).  Each
    shard's index list is returned in ascending order.
    """
    if num_ranks <= 0:
        raise ValueError("num_ranks must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, r) for r in range(num_ranks)]
    shards: list[list[int]] = [[] for _ in range(num_ranks)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(s) for s in shards]


def shard_loads(lengths: Sequence[int], shards: Sequence[Sequence[int]]) -> list[int]:
    return [sum(int(lengths[i]) for i in s) for s in shards]


_GATHER_INDEX: dict = {}


def _gather_index(shards, rows, device):
    """(source rows in the padded all-gather buffer, destination rows in the
    global batch) as device tensors, cached per shard layout and device."""
    import torch

    key = (tuple(tuple(int(i) for i in s) for s in shards), rows, str(device))
    idx = _GATHER_INDEX.get(key)
    if idx is None:
        src = [r * rows + j for r, s in enumerate(shards) for j in range(len(s))]
        dst = [int(i) for s in shards for i in s]
        idx = (torch.tensor(src, dtype=torch.int64, device=device),
               torch.tensor(dst, dtype=torch.int64, device=device))
        if len(_GATHER_INDEX) >= 64:
            _GATHER_INDEX.clear()
        _GATHER_INDEX[key] = idx
    return idx


def gather_outputs(local_out, shards, rank, group=None, dst=None):
    """Reassemble the global ``[B, Hq, D]`` output from per-rank shards.

    Every rank contributes its ``local_out`` (rows in the order of
    ``shards[rank]``); rows are padded to the largest shard and exchanged with
    one ``all_gather_into_tensor`` (NCCL over NVLink on GPUs, gloo on CPU).
    Returns the global tensor on every rank, or only on ``dst`` when given
    (``None`` elsewhere).  All ranks must call it (it is a collective).  The
    row permutation is one ``index_select`` + ``index_copy_`` with index
    tensors cached per shard layout, so a per-step call adds no host upload.
    """
    import torch
    import torch.distributed as dist

    world = len(shards)
    rows = max(len(s) for s in shards)
    total = sum(len(s) for s in shards)
    tail = tuple(local_out.shape[1:])
    if local_out.shape[0] == rows and local_out.is_contiguous():
        padded = local_out
    else:
        padded = local_out.new_zeros((rows, *tail))
        if local_out.shape[0]:
            padded[: local_out.shape[0]] = local_out
    if dist.get_backend(group) == "gloo":
        parts = [torch.empty_like(padded) for _ in range(world)]
        dist.all_gather(parts, padded, group=group)
        gathered = torch.stack(parts)
    else:
        gathered = padded.new_empty((world * rows, *tail))
        dist.all_gather_into_tensor(gathered, padded, group=group)
    if dst is not None and rank != dst:
        return None
    src_idx, dst_idx = _gather_index(shards, rows, local_out.device)
    out = local_out.new_empty((total, *tail))
    out.index_copy_(0, dst_idx, gathered.reshape(world * rows, *tail).index_select(0, src_idx))
    return out
