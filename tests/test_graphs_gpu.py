"""CUDA-graph forwards (``PagedLMMixin.enable_cuda_graphs``) vs eager forwards.

The graph path replays the same kernels on a batch padded to a bucket, so its
logits and stored K/V agree with the eager path to rounding (the padded GEMM
and the attention split plan may reduce in another order); the C1 reference
runs reproduce token for token with graphs on.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_json
from engine import workloads
from engine.attention import gather_ctx
from engine.config import EngineConfig, WorkloadRequest
from engine.qwen import build_random_model
from engine.scheduler import build_kv
from engine.spec_scheduler import SpeculativePagedScheduler
from engine.weights import qwen_numpy_state
from specdec.config import SamplingConfig as SpecSampling

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _model(name, seed, dtype=torch.float32):
    cfg = workloads.shape_config(name)
    state = {k: torch.from_numpy(v) for k, v in qwen_numpy_state(cfg, seed, 0.02).items()}
    return build_random_model(cfg, DEV, dtype, state_dict=state)


def _prefilled(model, prompts, max_seqs):
    kv = build_kv(model, EngineConfig(block_size=16, max_num_blocks=256), DEV, max_seqs=max_seqs)
    for sid, p in enumerate(prompts):
        kv.add_sequence(sid)
        model.prefill(torch.tensor([p], device=DEV), kv, [sid], [len(p)])
    return kv


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 5e-2)])
def test_graph_decode_and_block_match_eager(dtype, tol):
    eager = _model("c1-target", 1, dtype)
    graphed = _model("c1-target", 1, dtype)
    graphed.enable_cuda_graphs()
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 1024, size=int(n)).tolist() for n in (17, 40, 5)]
    kv_e = _prefilled(eager, prompts, max_seqs=3)
    kv_g = _prefilled(graphed, prompts, max_seqs=3)
    lens = [len(p) for p in prompts]
    for step in range(3):
        ids = torch.tensor(rng.integers(0, 1024, size=3), device=DEV)
        le = eager.decode(ids, kv_e, [0, 1, 2], lens)
        lg = graphed.decode(ids, kv_g, [0, 1, 2], lens)  # bucket 4: one padded row
        scale = le.float().abs().max().item()
        assert (le.float() - lg.float()).abs().max().item() <= tol * scale, step
        lens = [x + 1 for x in lens]
        if step == 1:  # more sequence rows than the table holds: the table moves, graphs recapture
            for kv in (kv_e, kv_g):
                for sid in range(3, 70):
                    kv.add_sequence(sid)
    block = torch.tensor(rng.integers(0, 1024, size=(3, 5)), device=DEV)
    be = eager.decode_block(block, kv_e, [0, 1, 2], lens)
    bg = graphed.decode_block(block, kv_g, [0, 1, 2], lens)
    assert be.shape == bg.shape == (3, 5, 1024)
    assert (be.float() - bg.float()).abs().max().item() <= tol * be.float().abs().max().item()
    for layer in range(eager.num_layers):
        a, b = kv_e._k[layer].float(), kv_g._k[layer].float()
        assert (a - b).abs().max().item() <= tol * a.abs().max().item()
    assert kv_e.block_tables == kv_g.block_tables
    kv_e.check_errors()
    kv_g.check_errors()


@pytest.mark.parametrize("label", ["greedy", "t1"])
def test_c1_runs_reproduce_with_graphs(label):
    g = load_json("c1_spec.json")
    run = g["runs"][label]
    C1 = workloads.C1
    target = _model("c1-target", C1["target_seed"])
    draft = _model("c1-draft", C1["draft_seed"])
    target.enable_cuda_graphs()
    draft.enable_cuda_graphs()
    cfg = EngineConfig(block_size=C1["block_size"], max_num_blocks=g["capacity"])
    kv = build_kv(target, cfg, DEV)
    dkv = build_kv(draft, cfg, DEV)
    sched = SpeculativePagedScheduler(target, kv, draft, dkv, cfg, SpecSampling(temperature=run["temperature"]),
                                      C1["gamma"], uniforms=torch.from_numpy(workloads.c1_uniforms(0)))
    reqs = [WorkloadRequest(prompt=ids, max_new_tokens=n, arrive_time=a) for ids, n, a in workloads.c1_requests(0)]
    res = sched.run_spec_continuous(reqs, seed=0, measure=False)
    assert [s.generated for s in res.sequences] == run["generated"]
    assert res.tokens_per_round == run["tokens_per_round"]
    kv.check_errors()
    dkv.check_errors()


def test_graph_prefill_matches_eager():
    """A 16-bit model with graphs on prefills a single prompt through a
    captured forward padded to a length bucket (64, then multiples of 128): first-token
    logits and the stored K/V agree with the eager prefill to bf16 rounding,
    on the capture, on a replay with another length in the same bucket and in
    a second bucket; fp32 models keep the eager prefill."""
    eager = _model("c1-target", 3, torch.bfloat16)
    graphed = _model("c1-target", 3, torch.bfloat16)
    graphed.enable_cuda_graphs()
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (40, 57, 130)]
    kvs = [build_kv(m, EngineConfig(block_size=16, max_num_blocks=256), DEV, max_seqs=4) for m in (eager, graphed)]
    for sid, p in enumerate(prompts):
        outs = []
        for m, kv in zip((eager, graphed), kvs):
            kv.add_sequence(sid)
            outs.append(m.prefill(torch.tensor([p], device=DEV), kv, [sid], [len(p)]).float())
        le, lg = outs
        assert le.shape == lg.shape == (1, 1024)
        assert (le - lg).abs().max().item() <= 5e-2 * le.abs().max().item(), sid
        for layer in (0, eager.num_layers - 1):
            ke = gather_ctx(kvs[0], layer, sid, len(p))
            kg = gather_ctx(kvs[1], layer, sid, len(p))
            for a, b in zip(ke, kg):
                assert (a.float() - b.float()).abs().max().item() <= 5e-2 * a.float().abs().max().item()
    assert kvs[0].block_tables == kvs[1].block_tables
    assert sorted(k[2] for k in graphed._graphs if k[1] == "prefill") == [64, 256]
    fp32 = _model("c1-target", 3)
    fp32.enable_cuda_graphs()
    kv32 = build_kv(fp32, EngineConfig(block_size=16, max_num_blocks=64), DEV, max_seqs=1)
    kv32.add_sequence(0)
    fp32.prefill(torch.tensor([prompts[0]], device=DEV), kv32, [0], [len(prompts[0])])
    assert not any(k[1] == "prefill" for k in getattr(fp32, "_graphs", {}))
    for kv in kvs + [kv32]:
        kv.check_errors()


@pytest.mark.parametrize("label", ["greedy", "t1"])
def test_precaptured_graphs_and_wall_clock_admission_reproduce_c1(label):
    """Every graph captured up front (``capture_graphs``, on a scratch
    sequence, before any request) and the wall-clock admission path with all
    arrivals at time 0: the C1 runs still reproduce the reference token for
    token and round for round, and the run captures nothing new."""
    g = load_json("c1_spec.json")
    run = g["runs"][label]
    C1 = workloads.C1
    target = _model("c1-target", C1["target_seed"])
    draft = _model("c1-draft", C1["draft_seed"])
    target.enable_cuda_graphs()
    draft.enable_cuda_graphs()
    cfg = EngineConfig(block_size=C1["block_size"], max_num_blocks=g["capacity"])
    kv = build_kv(target, cfg, DEV, max_seqs=16)
    dkv = build_kv(draft, cfg, DEV, max_seqs=16)
    sched = SpeculativePagedScheduler(target, kv, draft, dkv, cfg, SpecSampling(temperature=run["temperature"]),
                                      C1["gamma"], uniforms=torch.from_numpy(workloads.c1_uniforms(0)))
    n = sched.capture_graphs()
    spans = len(target.graph_spans(kv))
    # draft decode + target verify + the captured draft loops; fp32: no prefill graphs
    assert n == spans * len(target.GRAPH_BUCKETS) * 3
    assert kv.num_allocated_blocks == 0 and dkv.num_allocated_blocks == 0
    before = (len(target._graphs), len(draft._graphs))
    sched._next_sid = 0  # the scratch row is empty again: the run's sequence ids start at 0 as in the reference
    reqs = [WorkloadRequest(prompt=ids, max_new_tokens=n_, arrive_time=0.0)
            for ids, n_, _ in workloads.c1_requests(0)]
    rounds = []
    sched.round_hook = lambda sids, starts, d0: rounds.append(len(sids))
    res = sched.run_spec_continuous(reqs, seed=0, measure=False, arrival_clock="wall")
    assert [s.generated for s in res.sequences] == run["generated"]
    assert res.tokens_per_round == run["tokens_per_round"]
    assert (len(target._graphs), len(draft._graphs)) == before
    assert sched.round_replays == len(rounds) > 0  # every round was one whole-round replay
    kv.check_errors()
    dkv.check_errors()


def test_wall_clock_admission_waits_for_arrivals():
    """Requests arriving 0.3 s and 0.6 s into the run are admitted at a round
    boundary no earlier than their arrival; the run waits when idle."""
    import time as _time

    C1 = workloads.C1
    target = _model("c1-target", C1["target_seed"])
    draft = _model("c1-draft", C1["draft_seed"])
    cfg = EngineConfig(block_size=16, max_num_blocks=256)
    kv = build_kv(target, cfg, DEV)
    dkv = build_kv(draft, cfg, DEV)
    sched = SpeculativePagedScheduler(target, kv, draft, dkv, cfg, SpecSampling(temperature=0.0), C1["gamma"])
    reqs = [WorkloadRequest(prompt=ids, max_new_tokens=4, arrive_time=t)
            for (ids, _, _), t in zip(workloads.c1_requests(0)[:3], (0.0, 0.3, 0.6))]
    t0 = _time.perf_counter()
    res = sched.run_spec_continuous(reqs, seed=0, measure=True, arrival_clock="wall")
    assert _time.perf_counter() - t0 >= 0.6
    assert res.makespan_ms >= 600.0
    assert [len(s.generated) for s in res.sequences] == [4, 4, 4]
    assert [s.arrive_time for s in res.sequences] == [0.0, 0.3, 0.6]
    with pytest.raises(ValueError):
        sched.run_spec_continuous(reqs, seed=0, arrival_clock="tick")


def test_batched_chunked_prefill_matches_one_by_one():
    """``prefill_batch`` (prompts cut into 128-token chunks, one
    extend-attention row per chunk, each layer's K/V stored before it
    attends) gives the first-token logits and the stored K/V of one-by-one
    prefills to bf16 rounding, with the same block tables (reference
    allocation order)."""
    m = _model("c1-target", 3, torch.bfloat16)
    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (5, 128, 129, 300)]
    cfg = EngineConfig(block_size=16, max_num_blocks=256)
    kv1 = build_kv(m, cfg, DEV, max_seqs=4)
    kv2 = build_kv(m, cfg, DEV, max_seqs=4)
    one = []
    for sid, p in enumerate(prompts):
        kv1.add_sequence(sid)
        one.append(m.prefill(torch.tensor([p], device=DEV), kv1, [sid], [len(p)]).float())
    for sid in range(len(prompts)):
        kv2.add_sequence(sid)
    both = m.prefill_batch([prompts[0], torch.tensor(prompts[1], device=DEV)] + prompts[2:], kv2,
                           list(range(len(prompts)))).float()
    assert both.shape == (4, 1024)
    for sid in range(len(prompts)):
        a, b = one[sid][0], both[sid]
        assert (a - b).abs().max().item() <= 5e-2 * a.abs().max().item(), sid
        for layer in range(m.num_layers):
            ke = gather_ctx(kv1, layer, sid, len(prompts[sid]))
            kb = gather_ctx(kv2, layer, sid, len(prompts[sid]))
            for x, y in zip(ke, kb):
                assert (x.float() - y.float()).abs().max().item() <= 5e-2 * x.float().abs().max().item()
    assert kv1.block_tables == kv2.block_tables
    assert kv1.seq_lengths == kv2.seq_lengths
    kv1.check_errors()
    kv2.check_errors()


def test_graphed_batched_prefill_matches_eager():
    """``prefill_batch`` through the captured row-bucket graphs (rows past the
    call's repeat row 0 with nothing valid) gives the eager batched
    prefill's first-token logits and stored K/V to bf16 rounding, with the
    same block tables, and the precaptured graphs serve every row count."""
    g = torch.Generator().manual_seed(13)
    prompts = [torch.randint(0, 1024, (n,), generator=g).tolist() for n in (5, 128, 129, 300, 77)]
    cfg = EngineConfig(block_size=16, max_num_blocks=512)
    eager = _model("c1-target", 7, torch.bfloat16)
    graphed = _model("c1-target", 7, torch.bfloat16)
    graphed.enable_cuda_graphs()
    kv1 = build_kv(eager, cfg, DEV, max_seqs=8)
    kv2 = build_kv(graphed, cfg, DEV, max_seqs=8)
    kv2.add_sequence(0)
    graphed.capture_graphs(kv2, 0, 1, buckets=[1])
    n_rows = sum(1 for k in graphed._graphs if k[1] == "prefill_rows")
    assert n_rows == len(graphed.PREFILL_ROW_BUCKETS)
    for sid in range(1, 1 + len(prompts)):
        kv1.add_sequence(sid)
        kv2.add_sequence(sid)
    sids = list(range(1, 1 + len(prompts)))
    for part in (slice(0, 2), slice(2, 5)):
        a = eager.prefill_batch(prompts[part], kv1, sids[part]).float()
        b = graphed.prefill_batch(prompts[part], kv2, sids[part]).float()
        assert (a - b).abs().max().item() <= 5e-2 * a.abs().max().item()
    assert sum(1 for k in graphed._graphs if k[1] == "prefill_rows") == n_rows  # nothing captured on use
    for sid in sids:
        n = len(prompts[sid - 1])
        for layer in range(eager.num_layers):
            for x, y in zip(gather_ctx(kv1, layer, sid, n), gather_ctx(kv2, layer, sid, n)):
                assert (x.float() - y.float()).abs().max().item() <= 5e-2 * x.float().abs().max().item()
    # (the captures' scratch reservations reorder kv2's free list, so physical ids differ)
    assert kv1.seq_lengths[1:] == kv2.seq_lengths[1:]
    assert [len(t) for t in kv1.block_tables[1:]] == [len(t) for t in kv2.block_tables[1:]]
    kv1.check_errors()
    kv2.check_errors()


@pytest.mark.parametrize("temperature", [0.0, 1.0])
def test_captured_draft_loop_matches_step_by_step(temperature):
    """The draft phase as one captured loop (reserve, forward, head and draw
    for all gamma steps in one graph), and the whole round as one graph
    (that loop, the target's reserve and verify forward, the rejection
    sampling and the commit, padding rows inert), give the tokens, round
    structure, block tables and uniform consumption of the step-by-step
    path on 16-bit models."""
    runs = []
    for loops, whole in ((False, False), (True, False), (True, True)):
        target = _model("c1-target", 5, torch.bfloat16)
        draft = _model("c1-draft", 6, torch.bfloat16)
        target.enable_cuda_graphs()
        draft.enable_cuda_graphs()
        cfg = EngineConfig(block_size=16, max_num_blocks=512)
        kv = build_kv(target, cfg, DEV, max_seqs=16)
        dkv = build_kv(draft, cfg, DEV, max_seqs=16)
        sched = SpeculativePagedScheduler(target, kv, draft, dkv, cfg, SpecSampling(temperature=temperature), 4)
        sched.draft_loops = loops
        sched.round_graphs = whole
        sched.capture_graphs()
        assert bool(sched._loops) == loops
        sched._next_sid = 0
        g = torch.Generator().manual_seed(21)
        reqs = [WorkloadRequest(prompt=torch.randint(0, 1024, (int(n),), generator=g).tolist(), max_new_tokens=24,
                                arrive_time=float(i // 3))
                for i, n in enumerate((5, 40, 130, 17, 300, 64, 9))]
        rounds = []
        tables = []
        # (the captures' scratch reservations order each run's free lists
        # differently, so the tables are compared by their lengths)
        sched.round_hook = lambda sids, starts, d0: (rounds.append(len(sids)), tables.append(
            ([len(t) for t in kv.block_tables], [len(t) for t in dkv.block_tables], list(kv.seq_lengths),
             list(dkv.seq_lengths))))
        res = sched.run_spec_continuous(reqs, seed=3, measure=False)
        runs.append(([s.generated for s in res.sequences], res.tokens_per_round, res.draft_forward_calls,
                     rounds, tables, (sched.loop_replays, sched.round_replays)))
        kv.check_errors()
        dkv.check_errors()
    assert runs[0][:5] == runs[1][:5] == runs[2][:5]
    n = len(runs[0][3])
    assert n > 0 and runs[0][5] == (0, 0) and runs[1][5] == (n, 0) and runs[2][5] == (0, n)
