"""Sentence sharding across the GPUs of one node (one process per GPU).

Sentences are independent, so the attention path (and a translation built on
it) needs no collective on the data path: each rank takes a shard, runs it on
its own GPU with its own context, and the results are gathered once at the
end.  The reference translates one sentence per process (main.c:274-290);
this module is the batch layer above it.
"""
from __future__ import annotations

import heapq
from typing import List, Optional, Sequence


def decode_steps(n_src: int, max_gen: int) -> int:
    """Target steps the reference's beam search runs for a source of n_src
    tokens: min(3*n_src + 10, max_gen - 4) (main.c:315-316)."""
    return min(3 * n_src + 10, max_gen - 4)


BEAMS = 4
# Costs in units of one decoder row-step: one beam row through the 12 decoder
# layers' linear layers (14M weights each) and the tied vocabulary projection
# (262M), 424M multiply-adds, which the GEMMs stream for every step.
ENCODER_ROW = 0.34       # an encoder row: 12 layers of 12M weights = 144M multiply-adds
SELF_PER_POSITION = 7e-4  # 4 beams x 16 heads x 512 B of cache per position, at HBM speed
CROSS_PER_ROW = 1.8e-4    # 16 heads x 512 B of memory per source row, read once for all beams


def sentence_cost(n_src: int, max_gen: int) -> float:
    """Relative GPU work of one sentence in decoder row-steps: its encoder
    rows, then per decode step its beams' rows through the weights (the
    dominant term) plus the attention reads of that step (the cache so far
    and the encoder memory)."""
    steps = decode_steps(n_src, max_gen)
    attention = steps * (SELF_PER_POSITION * (steps + 1) / 2 + CROSS_PER_ROW * n_src)
    return ENCODER_ROW * n_src + BEAMS * steps + attention


def plan_shards(src_lengths: Sequence[int], world: int, max_gen: int = 132) -> List[List[int]]:
    """Longest-processing-time assignment of sentence indices to `world`
    ranks: sentences in decreasing cost order, each to the least-loaded rank.
    Deterministic (ties broken by index), so every rank computes the same plan
    without communicating.  Each shard lists its sentences in ascending index."""
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(src_lengths)),
                   key=lambda i: (-sentence_cost(int(src_lengths[i]), max_gen), i))
    heap = [(0, r) for r in range(world)]
    heapq.heapify(heap)
    shards: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + sentence_cost(int(src_lengths[i]), max_gen), r))
    return [sorted(s) for s in shards]


def shard_loads(src_lengths: Sequence[int], shards: Sequence[Sequence[int]], max_gen: int = 132) -> List[float]:
    return [sum(sentence_cost(int(src_lengths[i]), max_gen) for i in s) for s in shards]


def gather_results(local: dict, group=None) -> Optional[dict]:
    """Merge {sentence index: result} dicts of all ranks onto every rank (one
    all_gather_object after the work is done; the only collective)."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return dict(local)
    parts = [None] * dist.get_world_size(group)
    dist.all_gather_object(parts, local, group=group)
    merged: dict = {}
    for p in parts:
        overlap = merged.keys() & p.keys()
        if overlap:
            raise RuntimeError(f"sentences computed twice: {sorted(overlap)[:5]}")
        merged.update(p)
    return merged
