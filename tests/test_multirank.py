"""Host logic of the multi-GPU runner on CPU ranks (gloo, world size 2).

Requests are independent and weights replicated, so ranks exchange no
activations: each rank takes an LPT shard of the request set and the only
collectives are the barrier and the max / sum reductions of the timings that
bench.py performs. These tests run those steps on gloo ranks without a GPU,
including a rank that fails before the reduction.
"""
import os
import socket
import sys
from pathlib import Path

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, fail_rank):
    sys.path.insert(0, str(ROOT / "clef-rs_b200"))
    import torch
    from datetime import timedelta

    from clef_b200 import workloads
    from clef_b200.config import benchmark_config, flops_per_request
    from clef_b200.sharding import imbalance, lpt_assign, rank_shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        cfg = benchmark_config()
        batch = workloads.backbone_requests(n=256, seed=3)
        cost = lambda r: flops_per_request(cfg, len(r))  # noqa: E731
        mine = rank_shard(batch, rank, world, cost)
        ids = sorted(i for i, r in enumerate(batch) if any(r is m for m in mine))
        gathered = [None] * world
        dist.all_gather_object(gathered, ids)
        if rank == fail_rank:
            raise RuntimeError("injected rank failure before the timing reduction")
        t = torch.tensor([10.0 + rank], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        toks = torch.tensor([float(sum(len(m) for m in mine))], dtype=torch.float64)
        dist.all_reduce(toks, op=dist.ReduceOp.SUM)
        costs = [cost(r) for r in batch]
        q.put(("ok", rank, gathered, float(t.item()), float(toks.item()),
               imbalance(costs, lpt_assign(costs, world)), sum(len(r) for r in batch)))
    except Exception as e:  # reported to the parent, never hangs it
        q.put(("error", rank, repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_ranks_partition_requests_and_reduce_timings():
    out = _run(2)
    assert all(o[0] == "ok" for o in out), out
    _, _, gathered, tmax, toks, imb, total = out[0]
    flat = sorted(i for g in gathered for i in g)
    assert flat == list(range(256))          # every request exactly once
    assert tmax == 11.0                        # max over ranks
    assert toks == total                       # all tokens accounted for
    assert imb < 1.01                          # LPT balances the FLOP cost


def test_failed_rank_is_reported_not_hung():
    out = _run(2, fail_rank=1)
    kinds = {o[1]: o[0] for o in out}
    assert kinds[1] == "error"
    # The surviving rank's collective ends with an error (peer gone) rather than
    # waiting forever; the process-group timeout bounds the wait.
    assert kinds[0] in ("error", "ok")
    assert any("injected" in o[2] for o in out if o[0] == "error")


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
def test_lpt_balance_on_the_benchmark_batch(ranks):
    sys.path.insert(0, str(ROOT / "clef-rs_b200"))
    from clef_b200 import workloads
    from clef_b200.config import benchmark_config, flops_per_request
    from clef_b200.sharding import imbalance, lpt_assign
    cfg = benchmark_config()
    costs = [flops_per_request(cfg, len(r)) for r in workloads.backbone_requests(n=256, seed=3)]
    a = lpt_assign(costs, ranks)
    assert sorted(i for s in a for i in s) == list(range(256))
    assert imbalance(costs, a) < 1.02


class _FakePrefix:
    """Host stand-in for clef_b200.Prefix: its 'device allocation' is a CPU
    byte tensor, so the broadcast logic runs on gloo ranks."""

    def __init__(self, data):
        import torch
        self.data = torch.as_tensor(data, dtype=torch.uint8).clone()

    def span_bytes(self):
        return self.data.numel()

    def export_to(self, buf):
        buf.copy_(self.data)

    def import_from(self, buf):
        self.data.copy_(buf)


def _share_worker(rank, world, port, q):
    sys.path.insert(0, str(ROOT / "clef-rs_b200"))
    from datetime import timedelta

    import numpy as np

    from clef_b200.sharding import share_prefix
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        computed = []
        pattern = (np.arange(4096) * 7 % 251).astype(np.uint8)

        def compute():
            computed.append(rank)
            return _FakePrefix(pattern)

        p, cms, bms = share_prefix(compute, lambda: _FakePrefix(np.zeros(4096, np.uint8)), rank, world, "cpu")
        q.put(("ok", rank, computed, p.data.numpy().tobytes() == pattern.tobytes(), cms >= 0, bms is not None))
    except Exception as e:
        q.put(("error", rank, repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_prefix_is_computed_once_and_broadcast():
    """Config 5's prefix: rank 0 alone computes it, every rank ends with rank
    0's bytes (share_prefix, the logic bench.py runs over NCCL)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_share_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(3)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert all(o[0] == "ok" for o in out), out
    for _, rank, computed, same, ok_ms, has_bcast in out:
        assert computed == ([0] if rank == 0 else [])
        assert same and ok_ms and has_bcast


def _share_fail_worker(rank, world, port, q, mode):
    sys.path.insert(0, str(ROOT / "clef-rs_b200"))
    import time
    from datetime import timedelta

    import numpy as np

    from clef_b200.sharding import share_prefix
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    t0 = time.perf_counter()
    try:
        def compute():
            if mode == "compute_raises":
                raise ValueError("prefix prefill failed")
            return _FakePrefix(np.ones(4096, np.uint8))

        def create():
            n = 4096 + (16 if (mode == "span_differs" and rank == world - 1) else 0)
            return _FakePrefix(np.zeros(n, np.uint8))

        share_prefix(compute, create, rank, world, "cpu")
        q.put(("no error", rank, time.perf_counter() - t0, ""))
    except Exception as e:
        q.put(("raised", rank, time.perf_counter() - t0, str(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


@pytest.mark.parametrize("mode", ["span_differs", "compute_raises"])
def test_share_prefix_fails_on_every_rank_together(mode):
    """A layout that differs on one rank (rank 0 holding the largest span is
    the case a one-sided check misses) or a prefill that raises on rank 0: all
    ranks raise, promptly, instead of some waiting in the broadcast."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 3
    procs = [ctx.Process(target=_share_fail_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert sorted(o[1] for o in out) == list(range(world))
    for status, rank, seconds, msg in out:
        assert status == "raised", (rank, msg)
        assert seconds < 30, (rank, seconds)
        if mode == "span_differs":
            assert "disagree" in msg
        else:
            assert "failed on rank(s) [0]" in msg
