"""Pin the oracle schedulers to the reference's end-to-end runs (CPU only).

* C1 (Qwen2-shaped 2-layer target / 1-layer draft, numpy weights, gamma=4):
  greedy and T=1.0 with the injected uniform stream -- identical tokens,
  tokens_per_round, draft forward counts and the block tables of both caches
  after every round.
* The reference's committed toy goldens (results/cpu/*_correctness_toy.json).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_json
from engine import workloads
from engine.model import ToyConfig, ToyPagedLM, make_rotary_cache
from engine.weights import qwen_numpy_state
from oracle import kv as okv
from oracle import scheduler as osched
from oracle.model import NumpyPagedLM
from oracle.sampler import UniformStream


def _c1_models():
    C1 = workloads.C1
    out = []
    for name, seed in (("c1-target", C1["target_seed"]), ("c1-draft", C1["draft_seed"])):
        cfg = workloads.shape_config(name)
        rope = make_rotary_cache(cfg.head_dim, cfg.rope_theta, cfg.max_position_embeddings, torch.device("cpu"))
        out.append((cfg, NumpyPagedLM(qwen_numpy_state(cfg, seed, C1["weight_std"]), cfg.num_hidden_layers,
                                      cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim,
                                      rope.numpy(), kind="qwen")))
    return out


def _snapshot_hook(kv, dkv, snaps):
    return lambda: snaps.append({"target": [list(t) for t in kv.block_tables],
                                 "target_len": list(kv.seq_lengths),
                                 "draft": [list(t) for t in dkv.block_tables],
                                 "draft_len": list(dkv.seq_lengths)})


@pytest.mark.parametrize("label", ["greedy", "t1"])
def test_oracle_c1_spec_run_matches_reference(label):
    g = load_json("c1_spec.json")
    run = g["runs"][label]
    (tcfg, target), (dcfg, draft) = _c1_models()
    cap = g["capacity"]
    kv = okv.PagedKVCache(tcfg.num_hidden_layers, tcfg.num_key_value_heads, tcfg.head_dim, cap, 16)
    dkv = okv.PagedKVCache(dcfg.num_hidden_layers, dcfg.num_key_value_heads, dcfg.head_dim, cap, 16)
    reqs = [osched.Req(ids, n, a) for ids, n, a in workloads.c1_requests(0)]
    snaps = []
    hook = _snapshot_hook(kv, dkv, snaps)
    res = osched.run_spec_continuous(target, kv, draft, dkv, reqs, workloads.C1["gamma"], run["temperature"],
                                     stream=UniformStream(workloads.c1_uniforms(0)), round_hook=hook)
    assert [s.generated for s in res.sequences] == run["generated"]
    assert res.tokens_per_round == run["tokens_per_round"]
    assert res.steps == run["steps"]
    assert res.draft_forward_calls == run["draft_forward_calls"]
    assert res.kv_peak_blocks == run["kv_peak_blocks"]
    assert res.draft_kv_peak_blocks == run["draft_kv_peak_blocks"]
    assert snaps == run["snapshots"]


def _toy_numpy(cfg):
    m = ToyPagedLM(cfg, torch.device("cpu"))
    params = {k: v.detach().numpy() for k, v in m.state_dict().items()}
    return NumpyPagedLM(params, cfg.num_layers, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim,
                        m._cos_sin.numpy(), kind="toy")


def test_toy_weights_and_oracle_reproduce_committed_spec_golden():
    g = load_json("toy_correctness.json")["spec"]
    seed = g["seed"]
    tgt = _toy_numpy(ToyConfig(seed=seed, vocab_size=16))
    drf = _toy_numpy(ToyConfig(seed=7, hidden_size=48, num_layers=2, num_attention_heads=4, num_key_value_heads=2,
                               head_dim=12, vocab_size=16))
    kv = okv.PagedKVCache(2, 2, 16, g["max_num_blocks"], g["block_size"])
    dkv = okv.PagedKVCache(2, 2, 12, g["max_num_blocks"], g["block_size"])
    tok = ToyPagedLM(ToyConfig(seed=seed), torch.device("cpu")).tokenizer
    reqs = [osched.Req(tok.encode(r["prompt"]), r["max_new_tokens"], r["arrive_time"]) for r in g["requests"]]
    res = osched.run_spec_continuous(tgt, kv, drf, dkv, reqs, g["gamma"], 0.0)
    assert [s.generated for s in res.sequences] == g["generated"]
    assert res.tokens_per_round == g["tokens_per_round"]


def test_toy_weights_and_oracle_reproduce_committed_engine_golden():
    g = load_json("toy_correctness.json")["engine"]
    model = _toy_numpy(ToyConfig(seed=g["seed"]))
    kv = okv.PagedKVCache(2, 2, 16, g["max_num_blocks"], g["block_size"])
    tok = ToyPagedLM(ToyConfig(seed=g["seed"]), torch.device("cpu")).tokenizer
    reqs = [osched.Req(tok.encode(r["prompt"]), r["max_new_tokens"], r["arrive_time"]) for r in g["requests"]]
    res = osched.run_continuous(model, kv, reqs, 0.0)
    assert [s.generated for s in res.sequences] == g["generated"]


def test_build_workload_matches_reference_requests():
    from engine.config import DEFAULT_PROMPTS, WorkloadConfig, build_workload
    from engine.sampler import build_generator

    g = load_json("toy_correctness.json")["engine"]
    wl = WorkloadConfig(prompts=DEFAULT_PROMPTS, num_requests=6, min_tokens=4, max_tokens=16, arrival_window=4,
                        seed=g["seed"])
    reqs = build_workload(wl, build_generator(g["seed"]))
    assert [r.to_dict() for r in reqs] == g["requests"]
