"""Request sharding for data-parallel prefill over the GPUs of one box.

Requests are independent and weights are replicated, so ranks exchange no
activations: each rank takes a disjoint subset of requests chosen by the
longest-processing-time-first greedy rule (largest cost to the least-loaded
rank), with cost = the request's prefill FLOPs.
"""
import heapq
from typing import List, Sequence


def lpt_assign(costs: Sequence[float], ranks: int) -> List[List[int]]:
    if ranks <= 0:
        raise ValueError("ranks must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    heap = [(0.0, r) for r in range(ranks)]
    out: List[List[int]] = [[] for _ in range(ranks)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    for r in range(ranks):
        out[r].sort()
    return out


def shard_for(rank: int, ranks: int, costs: Sequence[float]) -> List[int]:
    return lpt_assign(costs, ranks)[rank]


def imbalance(costs: Sequence[float], assignment: List[List[int]]) -> float:
    loads = [sum(costs[i] for i in a) for a in assignment]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean else 1.0


def rank_shard(requests, rank: int, ranks: int, cost):
    """The requests rank `rank` of `ranks` serves: LPT over cost(request)."""
    if not 0 <= rank < ranks:
        raise ValueError("rank out of range")
    costs = [float(cost(r)) for r in requests]
    return [requests[i] for i in lpt_assign(costs, ranks)[rank]]
