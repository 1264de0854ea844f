"""Batch sharding across the GPUs of one node.

Decoding sequences are independent (each keeps its own SRAM, temp region, KV
cache and logits), so a batch splits into contiguous blocks of sequences, one
block per rank, with no data exchange while a step runs.  After each step the
ranks all-gather only the greedy token ids (B x int32), so every rank can see
the whole batch's tokens in sequence order.
"""
from __future__ import annotations


def shard(total: int, world: int, rank: int) -> range:
    """Sequence ids owned by `rank`: a contiguous block of total / world."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if total % world:
        raise ValueError(f"batch {total} does not split over {world} ranks")
    per = total // world
    return range(rank * per, (rank + 1) * per)


def gather_tokens(local, world: int, group=None):
    """All ranks' token tensors concatenated in rank (= sequence) order."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return local
    parts = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(parts, local, group=group)
    return torch.cat(parts)
