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


def share_prefix(compute, create, rank: int, world: int, device="cuda", sync=None):
    """The prefix state every rank continues from, computed once on rank 0 and
    handed to the other ranks (config 5: one shared prefix, suffixes sharded).

    compute() -> prefix runs on rank 0 only; create() -> prefix makes an empty
    prefix of the same layout on the other ranks (clef_b200.Engine.create_prefix
    with rank 0's token count and the same weights). Rank 0's device allocation
    then reaches them by one broadcast (torch.distributed, NCCL on GPUs): a
    prefix exposes span_bytes(), export_to(buf) and import_from(buf) like
    clef_b200.Prefix. `sync` (e.g. torch.cuda.synchronize) orders the copies
    around the broadcast. Returns (prefix, compute_ms, broadcast_ms or None)."""
    import time

    import torch
    import torch.distributed as dist
    sync = sync or (lambda: None)
    t0 = time.perf_counter()
    prefix = compute() if rank == 0 else create()
    sync()
    compute_ms = 1000 * (time.perf_counter() - t0)
    if world == 1:
        return prefix, compute_ms, None
    span = torch.tensor([prefix.span_bytes()], dtype=torch.int64, device=device)
    dist.all_reduce(span, op=dist.ReduceOp.MAX)
    if int(span.item()) != prefix.span_bytes():
        raise RuntimeError("share_prefix: ranks disagree on the prefix layout")
    buf = torch.empty(int(span.item()), dtype=torch.uint8, device=device)
    if rank == 0:
        prefix.export_to(buf)
    sync()
    dist.barrier()
    t1 = time.perf_counter()
    dist.broadcast(buf, src=0)
    sync()
    broadcast_ms = 1000 * (time.perf_counter() - t1)
    if rank != 0:
        prefix.import_from(buf)
    sync()
    return prefix, compute_ms, broadcast_ms
