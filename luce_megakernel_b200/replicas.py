"""Independent per-GPU replicas: the model is small and a token's forward is one dependent chain,
so multi-GPU runs are N processes with one GPU, their own weights copy and a disjoint request
stream each.  There is no collective on the data path; torch.distributed is used only to line the
ranks up for timing and to combine their counters.

The helpers below are the host-side logic of that mode (request assignment, timing barrier,
aggregation) and work with any backend: NCCL on GPUs, gloo in the CPU tests.
"""
from dataclasses import dataclass
from typing import List, Sequence


def assign_requests(num_requests: int, world_size: int, rank: int) -> List[int]:
    """Request ids served by `rank`: a round-robin split, disjoint across ranks and complete."""
    if world_size < 1 or not (0 <= rank < world_size):
        raise ValueError("bad rank / world_size")
    return list(range(rank, num_requests, world_size))


def request_seed(request_id: int) -> int:
    """Seed of a request's synthetic prompt (request i of a batch uses seed i)."""
    return int(request_id)


@dataclass
class ReplicaResult:
    tokens: int          # tokens this rank produced in the timed region
    seconds: float       # this rank's device time for the timed region


def aggregate(results: Sequence[ReplicaResult]) -> dict:
    """Whole-job throughput: all tokens divided by the slowest rank's time."""
    if not results:
        raise ValueError("no results")
    total = sum(r.tokens for r in results)
    slowest = max(r.seconds for r in results)
    return {"tokens": total, "seconds": slowest, "tokens_per_s": total / slowest if slowest > 0 else float("inf"),
            "n_replicas": len(results)}


def gather_results(local: ReplicaResult, group=None) -> List[ReplicaResult]:
    """All ranks' results on every rank (all_gather_object; off the data path)."""
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return [local]
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, (local.tokens, local.seconds), group=group)
    return [ReplicaResult(int(t), float(s)) for t, s in out]


def timing_barrier(device_sync=None, group=None):
    """Barrier + device synchronise on both sides of a timed region."""
    import torch.distributed as dist
    if device_sync is not None:
        device_sync()
    if dist.is_available() and dist.is_initialized():
        dist.barrier(group=group)
    if device_sync is not None:
        device_sync()
