"""Request sharding across the GPUs of one node (one process per GPU).

Sequences are independent -- own pages, own accept / rewind -- so the
speculative engine scales by giving every rank its own subset of requests,
its own KV pools and its own uniform stream.  Nothing is exchanged on the
data path; ``gather_results`` collects per-rank telemetry once at the end
(NCCL on GPUs, gloo on CPU), and ``merge`` aggregates it the way a single
``SchedulerResult`` would: generated tokens summed, makespan = slowest rank.
"""

from __future__ import annotations

import datetime
import os
from typing import Any, Dict, List, Optional, Sequence

import torch
import torch.distributed as dist


def rank_world() -> tuple:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1"))


def init_from_env(backend: Optional[str] = None, timeout_s: float = 120.0) -> tuple:
    """Initialise the default process group from torchrun's environment."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 and not dist.is_initialized():
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if backend is None:
            backend = "nccl" if torch.cuda.is_available() else "gloo"
        kw = {}
        if backend == "nccl":
            local = int(os.environ.get("LOCAL_RANK", "0"))
            torch.cuda.set_device(local)
            kw["device_id"] = torch.device("cuda", local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    return rank_world()


def shard_requests(requests: Sequence[Any], rank: int, world: int, policy: str = "round_robin") -> List[Any]:
    """The requests rank ``rank`` serves.

    ``round_robin`` (arrival-ordered streams, C4): request i goes to rank
    i % world.  ``contiguous`` (fixed batches, C2/C3/C5): equal consecutive
    slices, the remainder spread over the first ranks.
    """
    if world <= 1:
        return list(requests)
    if policy == "round_robin":
        return [r for i, r in enumerate(requests) if i % world == rank]
    if policy == "contiguous":
        n = len(requests)
        base, extra = divmod(n, world)
        lo = rank * base + min(rank, extra)
        hi = lo + base + (1 if rank < extra else 0)
        return list(requests[lo:hi])
    raise ValueError("unknown shard policy {}".format(policy))


def gather_results(payload: Dict[str, Any]) -> Optional[List[Dict[str, Any]]]:
    """All ranks' payloads on rank 0 (None elsewhere); identity when single-process."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return [payload]
    out: List[Optional[Dict[str, Any]]] = [None] * dist.get_world_size()
    dist.all_gather_object(out, payload)
    return out if dist.get_rank() == 0 else None


def merge(payloads: Sequence[Dict[str, Any]]) -> Dict[str, Any]:
    """Aggregate per-rank telemetry: tokens summed, makespan = slowest rank."""
    tokens = sum(int(p["generated_tokens"]) for p in payloads)
    makespan = max(float(p["makespan_ms"]) for p in payloads)
    tpr = [k for p in payloads for k in p.get("tokens_per_round", [])]
    return {
        "ranks": len(payloads),
        "generated_tokens": tokens,
        "makespan_ms": makespan,
        "throughput_tokens_per_s": tokens / (makespan / 1000.0) if makespan > 0 else None,
        "mean_tokens_per_round": (sum(tpr) / len(tpr)) if tpr else None,
    }
