"""The replica mode's host logic on two CPU ranks (gloo): disjoint request streams, timing
barrier, aggregation by the slowest rank.  No GPU involved."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from luce_megakernel_b200 import replicas as R


def test_assign_requests_is_a_partition():
    for n in (0, 1, 7, 16):
        for w in (1, 2, 4, 8):
            parts = [R.assign_requests(n, w, r) for r in range(w)]
            flat = sorted(x for p in parts for x in p)
            assert flat == list(range(n))
            assert max(len(p) for p in parts) - min(len(p) for p in parts) <= 1
    with pytest.raises(ValueError):
        R.assign_requests(4, 2, 2)


def test_aggregate_uses_slowest_rank():
    agg = R.aggregate([R.ReplicaResult(128, 0.10), R.ReplicaResult(128, 0.20)])
    assert agg["tokens"] == 256 and agg["seconds"] == 0.20 and abs(agg["tokens_per_s"] - 1280.0) < 1e-9


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = R.assign_requests(10, world, rank)
        # a fake decode loop: each request "produces" 4 tokens; rank 1 is slower
        R.timing_barrier()
        tokens = 4 * len(mine)
        seconds = 0.01 * (rank + 1)
        R.timing_barrier()
        allr = R.gather_results(R.ReplicaResult(tokens, seconds))
        agg = R.aggregate(allr)
        seeds = [R.request_seed(i) for i in mine]
        q.put((rank, mine, seeds, agg))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_replicas():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = sorted(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, m0, s0, a0), (r1, m1, s1, a1) = out
    assert set(m0).isdisjoint(m1) and sorted(m0 + m1) == list(range(10))
    assert s0 == m0 and s1 == m1
    assert a0 == a1                                   # every rank sees the same aggregate
    assert a0["tokens"] == 40 and abs(a0["seconds"] - 0.02) < 1e-12 and a0["n_replicas"] == 2
