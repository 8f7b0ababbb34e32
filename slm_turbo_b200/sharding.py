"""Host-side partitioning of decode work across GPUs (one process per GPU).

Decode attention of different sequences, and of different KV heads of one
sequence, is independent, so multi-GPU runs shard the units on the host and
need no collective on the data path.
"""
from __future__ import annotations

import heapq
from typing import List, Sequence


def partition_sequences(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Greedy longest-first bin packing of sequences onto ``world`` ranks by
    token count.  Returns, per rank, the sorted indices of its sequences.
    Deterministic: ties go to the lower rank."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    heap = [(0, r) for r in range(world)]
    parts: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(p) for p in parts]


def shard_kv_heads(num_kv_heads: int, world: int, rank: int) -> range:
    """KV heads owned by ``rank`` when the heads of long sequences are split
    across ``world`` GPUs (contiguous, equal shares)."""
    if num_kv_heads % world != 0:
        raise ValueError(f"{num_kv_heads} kv heads do not split over {world} ranks")
    per = num_kv_heads // world
    return range(rank * per, (rank + 1) * per)
