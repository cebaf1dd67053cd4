"""Request sharding + final gather across 2 gloo ranks on CPU.

Each rank runs the oracle speculative scheduler (C1 models, greedy) on its
shard with its own caches; rank 0 gathers the token streams.  Sequences are
independent, so the union must equal one process serving every request.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from engine import workloads
from engine.distributed import gather_results, merge, shard_requests


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _c1_oracle():
    from engine.model import make_rotary_cache
    from engine.weights import qwen_numpy_state
    from oracle.model import NumpyPagedLM

    C1 = workloads.C1
    out = []
    for name, seed in (("c1-target", C1["target_seed"]), ("c1-draft", C1["draft_seed"])):
        cfg = workloads.shape_config(name)
        rope = make_rotary_cache(cfg.head_dim, cfg.rope_theta, cfg.max_position_embeddings, torch.device("cpu"))
        out.append(NumpyPagedLM(qwen_numpy_state(cfg, seed, C1["weight_std"]), cfg.num_hidden_layers,
                                cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, rope.numpy()))
    return out


def _serve(reqs):
    from oracle import kv as okv
    from oracle import scheduler as osched

    target, draft = _c1_oracle()
    kv = okv.PagedKVCache(2, 2, 64, 64, 16)
    dkv = okv.PagedKVCache(1, 2, 64, 64, 16)
    res = osched.run_spec_continuous(target, kv, draft, dkv, [osched.Req(i, n, a) for i, n, a in reqs],
                                     workloads.C1["gamma"], 0.0)
    return res


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        reqs = [(ids, 12, 0) for ids, _, _ in workloads.c1_requests(0)]
        mine = shard_requests(list(enumerate(reqs)), rank, world, "round_robin")
        res = _serve([r for _, r in mine])
        payload = {"rank": rank, "ids": [i for i, _ in mine], "generated": [s.generated for s in res.sequences],
                   "generated_tokens": sum(len(s.generated) for s in res.sequences), "makespan_ms": 1.0 + rank,
                   "tokens_per_round": res.tokens_per_round}
        got = gather_results(payload)
        if rank == 0:
            q.put(got)
    finally:
        dist.destroy_process_group()


def test_shard_policies_partition_the_requests():
    reqs = list(range(10))
    for policy in ("round_robin", "contiguous"):
        parts = [shard_requests(reqs, r, 3, policy) for r in range(3)]
        assert sorted(x for p in parts for x in p) == reqs
        assert max(len(p) for p in parts) - min(len(p) for p in parts) <= 1


def test_two_gloo_ranks_reproduce_single_process_tokens():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    by_id = {}
    for payload in got:
        for i, g in zip(payload["ids"], payload["generated"]):
            by_id[i] = g
    reqs = [(ids, 12, 0) for ids, _, _ in workloads.c1_requests(0)]
    single = _serve(reqs)
    assert [by_id[i] for i in range(len(reqs))] == [s.generated for s in single.sequences]
    m = merge(got)
    assert m["ranks"] == 2 and m["generated_tokens"] == 12 * len(reqs) and m["makespan_ms"] == 2.0
