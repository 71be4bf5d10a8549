"""Sequence sharding across GPUs: one process per GPU, no collective on the path.

Every sequence's pages, block-table row and attention are self-contained (the
reference attends per request with no cross-request terms,
microinfer/layer/paged_attention.py:41-65), so a batch splits across ranks by
sequence: each rank owns its own KV pool (rank-local block ids) and its
subset of requests, and runs the unchanged single-GPU path.  The only
exchange is after sampling: every rank's token ids are gathered so the
scheduler sees the whole batch (NCCL over NVLink on GPUs, gloo on CPU).
"""

from __future__ import annotations

import heapq

import torch
import torch.distributed as dist


def assign_sequences(contexts, world_size: int) -> list[list[int]]:
    """Balance sequences over ranks by total context (the decode bytes).

    Longest-first greedy onto the currently lightest rank; ties go to the
    lower rank, so the assignment is deterministic on every rank.  Returns,
    per rank, the sequence indices in ascending order.
    """
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    contexts = [int(c) for c in contexts]
    if any(c < 0 for c in contexts):
        raise ValueError("contexts must be non-negative")
    heap = [(0, r) for r in range(world_size)]
    out: list[list[int]] = [[] for _ in range(world_size)]
    for idx in sorted(range(len(contexts)), key=lambda i: (-contexts[i], i)):
        load, rank = heapq.heappop(heap)
        out[rank].append(idx)
        heapq.heappush(heap, (load + contexts[idx], rank))
    return [sorted(v) for v in out]


def gather_tokens(local_tokens: torch.Tensor, assignment: list[list[int]], group=None) -> torch.Tensor:
    """All-gather per-rank sampled token ids back into global sequence order.

    ``local_tokens[i]`` is the token of sequence ``assignment[rank][i]``.
    Every rank pads to the largest shard, so all ranks issue the same
    collective with the same shape.
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if len(assignment) != world:
        raise ValueError("assignment must have one entry per rank")
    if local_tokens.numel() != len(assignment[rank]):
        raise ValueError("local_tokens does not match this rank's shard")
    width = max((len(a) for a in assignment), default=0)
    padded = torch.full((width,), -1, dtype=torch.int32, device=local_tokens.device)
    padded[: local_tokens.numel()] = local_tokens.to(torch.int32)
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    total = sum(len(a) for a in assignment)
    out = torch.full((total,), -1, dtype=torch.int32, device=local_tokens.device)
    for r, seqs in enumerate(assignment):
        if seqs:
            out[torch.tensor(seqs, device=out.device)] = parts[r][: len(seqs)]
    return out
