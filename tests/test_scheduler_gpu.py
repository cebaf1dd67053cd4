"""End-to-end schedulers on the GPU vs the reference's own runs.

* C1 (Qwen2-shaped fp32 models with the fixture's numpy weights, gamma=4):
  greedy and T=1.0 with the same injected uniform stream -- identical token
  streams, tokens_per_round, draft forward counts, KV peaks and the block
  tables of both caches after every round.
* The reference's committed toy goldens (spec and plain engine).
* The reference's scheduler tests restated: greedy spec == plain continuous,
  determinism, static == continuous.
"""

from __future__ import annotations

import copy

import pytest
import torch

from conftest import load_json
from engine import workloads
from engine.config import DEFAULT_PROMPTS, EngineConfig, SamplingConfig, WorkloadConfig, WorkloadRequest, build_workload
from engine.model import ToyConfig, ToyPagedLM
from engine.qwen import build_random_model
from engine.sampler import build_generator
from engine.scheduler import PagedScheduler, build_kv
from engine.spec_scheduler import SpeculativePagedScheduler
from engine.weights import qwen_numpy_state
from specdec.config import SamplingConfig as SpecSampling

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _c1_model(name, seed):
    cfg = workloads.shape_config(name)
    state = {k: torch.from_numpy(v) for k, v in qwen_numpy_state(cfg, seed, workloads.C1["weight_std"]).items()}
    return build_random_model(cfg, DEV, torch.float32, state_dict=state)


@pytest.mark.parametrize("label", ["greedy", "t1"])
def test_c1_spec_run_matches_reference(label, monkeypatch):
    g = load_json("c1_spec.json")
    run = g["runs"][label]
    C1 = workloads.C1
    target = _c1_model("c1-target", C1["target_seed"])
    draft = _c1_model("c1-draft", C1["draft_seed"])
    cfg = EngineConfig(block_size=C1["block_size"], max_num_blocks=g["capacity"])
    kv = build_kv(target, cfg, DEV)
    dkv = build_kv(draft, cfg, DEV)
    sched = SpeculativePagedScheduler(target, kv, draft, dkv, cfg, SpecSampling(temperature=run["temperature"]),
                                      C1["gamma"], uniforms=torch.from_numpy(workloads.c1_uniforms(0)))
    snaps = []
    orig = SpeculativePagedScheduler._spec_step

    def step_and_snap(self, running, result, stream):
        orig(self, running, result, stream)
        snaps.append({"target": copy.deepcopy(self.kv.block_tables), "target_len": list(self.kv.seq_lengths),
                      "draft": copy.deepcopy(self.draft_kv.block_tables), "draft_len": list(self.draft_kv.seq_lengths)})

    monkeypatch.setattr(SpeculativePagedScheduler, "_spec_step", step_and_snap)
    reqs = [WorkloadRequest(prompt=ids, max_new_tokens=n, arrive_time=a) for ids, n, a in workloads.c1_requests(0)]
    res = sched.run_spec_continuous(reqs, seed=0, measure=False)
    assert [s.generated for s in res.sequences] == run["generated"]
    assert res.tokens_per_round == run["tokens_per_round"]
    assert res.steps == run["steps"]
    assert res.draft_forward_calls == run["draft_forward_calls"]
    assert res.kv_peak_blocks == run["kv_peak_blocks"]
    assert res.draft_kv_peak_blocks == run["draft_kv_peak_blocks"]
    assert snaps == run["snapshots"]
    kv.check_errors()
    dkv.check_errors()


def test_committed_toy_spec_golden():
    g = load_json("toy_correctness.json")["spec"]
    seed = g["seed"]
    tgt = ToyPagedLM(ToyConfig(seed=seed, vocab_size=16), DEV)
    drf = ToyPagedLM(ToyConfig(seed=7, hidden_size=48, num_layers=2, num_attention_heads=4, num_key_value_heads=2,
                               head_dim=12, vocab_size=16), DEV)
    cfg = EngineConfig(block_size=g["block_size"], max_num_blocks=g["max_num_blocks"])
    sched = SpeculativePagedScheduler(tgt, build_kv(tgt, cfg, DEV), drf, build_kv(drf, cfg, DEV), cfg,
                                      SpecSampling(temperature=0.0), g["gamma"])
    reqs = [WorkloadRequest(**r) for r in g["requests"]]
    res = sched.run_spec_continuous(reqs, seed=seed, measure=False)
    assert [s.generated for s in res.sequences] == g["generated"]
    assert res.tokens_per_round == g["tokens_per_round"]


def test_committed_toy_engine_golden():
    g = load_json("toy_correctness.json")["engine"]
    model = ToyPagedLM(ToyConfig(seed=g["seed"]), DEV)
    cfg = EngineConfig(block_size=g["block_size"], max_num_blocks=g["max_num_blocks"])
    res = PagedScheduler(model, build_kv(model, cfg, DEV), cfg, SamplingConfig(temperature=0.0)).run_continuous(
        [WorkloadRequest(**r) for r in g["requests"]], seed=g["seed"], measure=False)
    assert [s.generated for s in res.sequences] == g["generated"]


def _workload(seed, n=4, lo=4, hi=10):
    wl = WorkloadConfig(prompts=DEFAULT_PROMPTS[:3], num_requests=n, min_tokens=lo, max_tokens=hi, arrival_window=2,
                        seed=seed)
    return build_workload(wl, build_generator(seed))


def test_spec_greedy_equals_plain_continuous():
    target = ToyPagedLM(ToyConfig(seed=0), DEV)
    draft = ToyPagedLM(ToyConfig(seed=7), DEV)
    cfg = EngineConfig(block_size=4, max_num_blocks=128)
    greedy = SamplingConfig(temperature=0.0)
    requests = _workload(1)
    base = PagedScheduler(target, build_kv(target, cfg, DEV), cfg, greedy).run_continuous(requests, seed=1)
    spec = SpeculativePagedScheduler(target, build_kv(target, cfg, DEV), draft, build_kv(draft, cfg, DEV), cfg,
                                     greedy, 2).run_spec_continuous(requests, seed=1)
    assert spec.mode == "spec-continuous"
    assert sorted((s.max_new_tokens, tuple(s.generated)) for s in base.sequences) == \
        sorted((s.max_new_tokens, tuple(s.generated)) for s in spec.sequences)
    assert all(s.finished for s in spec.sequences)


def test_spec_with_identical_draft_accepts_everything_and_catches_up():
    target = ToyPagedLM(ToyConfig(seed=0), DEV)
    draft = ToyPagedLM(ToyConfig(seed=0), DEV)
    cfg = EngineConfig(block_size=4, max_num_blocks=128)
    greedy = SamplingConfig(temperature=0.0)
    requests = _workload(3, n=5, lo=9, hi=16)
    base = PagedScheduler(target, build_kv(target, cfg, DEV), cfg, greedy).run_continuous(requests, seed=3)
    kv, dkv = build_kv(target, cfg, DEV), build_kv(draft, cfg, DEV)
    spec = SpeculativePagedScheduler(target, kv, draft, dkv, cfg, greedy, 3).run_spec_continuous(requests, seed=3)
    assert sorted(tuple(s.generated) for s in base.sequences) == sorted(tuple(s.generated) for s in spec.sequences)
    assert max(spec.tokens_per_round) == 4
    assert kv.num_allocated_blocks == 0 and dkv.num_allocated_blocks == 0
    assert len(kv.device_state()["free_list"]) == kv.capacity


def test_spec_is_deterministic():
    draft = ToyPagedLM(ToyConfig(seed=7), DEV)
    cfg = EngineConfig(block_size=4, max_num_blocks=128)
    requests = _workload(5)

    def run():
        target = ToyPagedLM(ToyConfig(seed=0), DEV)
        res = SpeculativePagedScheduler(target, build_kv(target, cfg, DEV), draft, build_kv(draft, cfg, DEV), cfg,
                                        SpecSampling(temperature=1.0), 2).run_spec_continuous(requests, seed=5)
        return [tuple(s.generated) for s in res.sequences], res.tokens_per_round

    assert run() == run()


def test_static_greedy_matches_continuous_and_metrics():
    model = ToyPagedLM(ToyConfig(seed=0), DEV)
    cfg = EngineConfig(block_size=4, max_num_blocks=64)
    requests = _workload(1, n=5, lo=3, hi=6)
    sampling = SamplingConfig(temperature=0.0)
    kv = build_kv(model, cfg, DEV)
    cont = PagedScheduler(model, kv, cfg, sampling).run_continuous(requests, seed=1)
    kv.reset()
    stat = PagedScheduler(model, kv, cfg, sampling).run_static(requests, seed=1)
    fp = lambda r: sorted((s.max_new_tokens, tuple(s.generated)) for s in r.sequences)  # noqa: E731
    assert fp(cont) == fp(stat)
    payload = cont.to_dict()
    assert payload["generated_tokens"] > 0 and payload["steps"] >= 1
    assert payload["throughput_tokens_per_s"] is not None
    assert 0.0 < payload["slot_utilization"] <= 1.0


def test_recompute_preemption_serves_c1_in_a_small_pool():
    """A pool too small for the C1 batch: the reference's policy raises
    BlockExhaustedError; the recompute policy admits what fits, parks the
    most recently admitted sequences before a round that would not fit,
    re-prefills them later, and finishes every request with the greedy
    tokens of the roomy run (recomputed K/V hold the same values)."""
    from engine.kv import BlockExhaustedError

    g = load_json("c1_spec.json")
    run = g["runs"]["greedy"]
    C1 = workloads.C1
    target = _c1_model("c1-target", C1["target_seed"])
    draft = _c1_model("c1-draft", C1["draft_seed"])
    reqs = [WorkloadRequest(prompt=ids, max_new_tokens=n, arrive_time=a) for ids, n, a in workloads.c1_requests(0)]

    def make(policy, blocks):
        cfg = EngineConfig(block_size=C1["block_size"], max_num_blocks=blocks)
        sched = SpeculativePagedScheduler(target, build_kv(target, cfg, DEV), draft, build_kv(draft, cfg, DEV), cfg,
                                          SpecSampling(temperature=0.0), C1["gamma"])
        sched.preemption = policy
        return sched

    with pytest.raises(BlockExhaustedError):
        make("raise", 20).run_spec_continuous(reqs, seed=0, measure=False)
    sched = make("recompute", 20)
    res = sched.run_spec_continuous(reqs, seed=0, measure=False)
    assert sched.preemptions > 0
    assert [s.generated for s in res.sequences] == run["generated"]
    assert sched.kv.num_allocated_blocks == 0 and sched.draft_kv.num_allocated_blocks == 0
    sched.kv.check_errors()
    sched.draft_kv.check_errors()
    # a single request larger than the whole pool cannot be served either way
    with pytest.raises(BlockExhaustedError):
        make("recompute", 3).run_spec_continuous(reqs[:1], seed=0, measure=False)
