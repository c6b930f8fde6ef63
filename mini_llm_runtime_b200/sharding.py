"""Request sharding of the paged hot path across GPUs (one process per GPU).

Decode and chunk-prefill requests are independent: every request reads only
its own blocks of the KV pool.  A multi-GPU batch is therefore split by
request, each rank keeping its requests' KV blocks in its own pool, with no
collective on the data path (the reference runs one process and one device:
runtime/model_runner.py:146-288 executes the whole ModelBatch in place).

The cost of a request is proportional to the KV it streams (decode) or the
query x key pairs it computes (prefill), so shards are balanced on that cost
rather than on request count: longest-processing-time-first greedy, each
request going to the currently lightest rank (ties to the lowest rank, so
every rank computes the same assignment from the same metadata without
communicating).
"""

from __future__ import annotations

import heapq
from dataclasses import dataclass, field
from typing import Sequence


@dataclass
class Shard:
    rank: int
    requests: list[int] = field(default_factory=list)  # indices into the global batch, ascending
    cost: int = 0


def decode_cost(context_len: int) -> int:
    """KV tokens a decode request streams."""
    return int(context_len)


def prefill_cost(prefix_len: int, chunk_len: int) -> int:
    """Query x key pairs of a causal chunk: chunk * (prefix + 1) + chunk * (chunk - 1) / 2."""
    c, p = int(chunk_len), int(prefix_len)
    return c * (p + 1) + c * (c - 1) // 2


def shard_requests(costs: Sequence[int], world_size: int) -> list[Shard]:
    """Split requests over ``world_size`` ranks, balancing total cost.

    Deterministic: the same costs give the same shards on every rank.
    Requests keep their global order inside a shard.
    """
    if world_size <= 0:
        raise ValueError("world_size must be positive")
    costs = [int(c) for c in costs]
    if any(c < 0 for c in costs):
        raise ValueError("request costs must be non-negative")
    shards = [Shard(rank=r) for r in range(world_size)]
    heap = [(0, r) for r in range(world_size)]
    heapq.heapify(heap)
    for i in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        load, r = heapq.heappop(heap)
        shards[r].requests.append(i)
        shards[r].cost += costs[i]
        heapq.heappush(heap, (load + costs[i], r))
    for s in shards:
        s.requests.sort()
    return shards


def imbalance(shards: Sequence[Shard]) -> float:
    """max rank cost / mean rank cost (1.0 = perfect balance)."""
    total = sum(s.cost for s in shards)
    if total == 0:
        return 1.0
    return max(s.cost for s in shards) / (total / len(shards))
