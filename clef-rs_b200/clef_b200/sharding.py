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
    around the broadcast. Returns (prefix, compute_ms, broadcast_ms or None).

    Every rank takes the same collective steps and the same decision: one
    all_gather of (ok, span) from all ranks, after which either every rank
    goes on to the broadcast or every rank raises (a failed compute() or
    create() on any rank, or ranks whose prefix layouts differ), so no rank is
    left waiting in a collective that the others never enter."""
    import time

    import torch
    import torch.distributed as dist
    sync = sync or (lambda: None)
    t0 = time.perf_counter()
    prefix, error = None, None
    try:
        prefix = compute() if rank == 0 else create()
        sync()
    except Exception as e:  # reported on every rank after the exchange below
        error = e
    compute_ms = 1000 * (time.perf_counter() - t0)
    if world == 1:
        if error is not None:
            raise error
        return prefix, compute_ms, None
    mine = torch.tensor([0 if error is not None else 1,
                         prefix.span_bytes() if error is None else -1], dtype=torch.int64, device=device)
    every = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(every, mine)
    table = [(int(t[0].item()), int(t[1].item())) for t in every]
    failed = [r for r, (ok, _) in enumerate(table) if not ok]
    if failed:
        why = f" ({error!r})" if error is not None else ""
        raise RuntimeError(f"share_prefix: prefix set-up failed on rank(s) {failed}{why}")
    spans = {span for _, span in table}
    if len(spans) != 1:
        raise RuntimeError(f"share_prefix: ranks disagree on the prefix layout (span bytes per rank "
                           f"{[span for _, span in table]})")
    span = spans.pop()
    buf = torch.empty(span, dtype=torch.uint8, device=device)
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
