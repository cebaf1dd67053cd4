"""Generate the golden fixtures in this directory from the reference itself.

Run in a container that has the reference checked out (it is imported, never
copied):  ``python tests/golden/make_golden.py --reference /path/to/speculative-decoding-lab``

Everything is computed by the reference's own CPU code on seeded inputs and
stored as small JSON / npz files.  The fixtures pin both the numpy oracle
(``oracle/``) and the CUDA path.  Stochastic draws go through one injected
uniform stream: the reference's ``_draw_uniform`` and ``sample_token`` (and
``PagedScheduler._sample``) are replaced by readers of that stream, and the
draw itself uses the defined integer inverse-CDF rule of ``oracle.sampler``.

Files written:
  kv_trace.json        scripted allocator / cache operations and every state
  attention.npz        decode / extend / prefill inputs and reference outputs
                       (fp32, and bf16 run through the reference's bf16 path)
  sampler.json         logits_to_probs rows, residual rows, batch_accept KATs
                       and stochastic cases with injected uniforms
  c1_spec.json         C1 runs (greedy and T=1.0): tokens, tokens_per_round,
                       per-round block tables of both caches
  toy_correctness.json the reference's committed toy goldens
                       (results/cpu/{spec,engine}_correctness_toy.json) with
                       the settings that reproduce them
"""

from __future__ import annotations

import argparse
import copy
import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _load_by_path(name: str, path: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SDL_REFERENCE"), required="SDL_REFERENCE" not in os.environ,
                    help="checkout of the reference project (or set SDL_REFERENCE)")
    args = ap.parse_args(argv)
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.reference)
    sys.path.insert(0, REPO)  # for `oracle`
    import torch

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    from engine import attention as ref_attn  # the reference's engine package
    from engine import kv as ref_kv
    from engine import scheduler as ref_sched
    from engine import spec_scheduler as ref_spec
    from engine.config import EngineConfig, WorkloadConfig, WorkloadRequest, build_workload
    from engine.config import DEFAULT_PROMPTS as ENGINE_PROMPTS
    from engine.model import ToyConfig, ToyPagedLM
    from engine.qwen import QwenPagedModel
    from engine.sampler import build_generator
    from specdec import sampler as ref_sampler
    from specdec.config import SamplingConfig as SpecSampling

    from oracle.sampler import sample_index

    pkg = os.path.join(REPO, "speculative-decoding-lab_b200", "engine")
    workloads = _load_by_path("sdl_workloads", os.path.join(pkg, "workloads.py"))
    weights = _load_by_path("sdl_weights", os.path.join(pkg, "weights.py"))

    # ---------------------------------------------------------- kv trace
    def kv_state(kv):
        return {
            "block_tables": copy.deepcopy(kv.block_tables),
            "seq_lengths": list(kv.seq_lengths),
            "num_allocated": kv.num_allocated_blocks,
            "free_list": list(kv.allocator._free),
        }

    kv = ref_kv.PagedKVCache(2, 2, 8, 16, 4, torch.device("cpu"), torch.float32)
    ops = []
    rng = np.random.default_rng(7)
    script = [("add", 0), ("add", 1), ("add", 2)]
    for pos in range(10):
        script.append(("write", 0, pos))
    for pos in range(6):
        script.append(("write", 1, pos))
    script += [("truncate", 0, 3), ("write", 2, 4), ("truncate", 1, 5), ("clear", 0),
               ("write", 1, 9), ("write", 0, 0), ("write", 2, 11), ("truncate", 2, 0), ("truncate", 1, 12),
               ("clear", 1), ("add", 4), ("write", 4, 2)]
    for pos in range(3, 14):
        script.append(("write", 4, pos))
    script += [("truncate", 4, 7), ("write", 3, 0), ("reset",)]
    for op in script:
        if op[0] == "add":
            kv.add_sequence(op[1])
        elif op[0] == "write":
            vec = torch.from_numpy(rng.standard_normal((2, 8)).astype(np.float32))
            kv.write(0, op[1], op[2], vec, vec)
        elif op[0] == "truncate":
            kv.truncate(op[1], op[2])
        elif op[0] == "clear":
            kv.clear(op[1])
        elif op[0] == "reset":
            kv.reset()
        ops.append({"op": list(op), "state": kv_state(kv)})
    exhaust = ref_kv.PagedKVCache(1, 1, 8, 3, 4, torch.device("cpu"), torch.float32)
    exhaust.add_sequence(0)
    for pos in range(12):
        exhaust.write(0, 0, pos, torch.zeros(1, 8), torch.zeros(1, 8))
    raised = False
    try:
        exhaust.write(0, 0, 12, torch.zeros(1, 8), torch.zeros(1, 8))
    except ref_kv.BlockExhaustedError as e:
        raised = str(e)
    with open(os.path.join(HERE, "kv_trace.json"), "w") as f:
        json.dump({"config": {"num_layers": 2, "num_kv_heads": 2, "head_dim": 8, "capacity": 16, "block_size": 4},
                   "ops": ops, "exhaustion_message": raised}, f)

    # ---------------------------------------------------------- attention
    arrays = {}

    def attn_case(tag, dtype, Hq, Hkv, d, bs, lens, chunk, seed):
        g = torch.Generator().manual_seed(seed)
        cap = sum((ln + chunk + bs - 1) // bs for ln in lens) + 4
        kvc = ref_kv.PagedKVCache(1, Hkv, d, cap, bs, torch.device("cpu"), dtype)
        total = [ln + chunk for ln in lens]
        for sid, T in enumerate(total):
            kvc.add_sequence(sid)
            k = torch.randn(T, Hkv, d, generator=g).to(dtype)
            v = torch.randn(T, Hkv, d, generator=g).to(dtype)
            for pos in range(T):
                kvc.write(0, sid, pos, k[pos], v[pos])
        B = len(lens)
        q = torch.randn(B, chunk, Hq, d, generator=g).to(dtype)
        if chunk == 1:
            out = ref_attn.paged_attention_decode(q[:, 0], kvc, 0, list(range(B)), total, Hq).unsqueeze(1)
            starts = [T - 1 for T in total]
        else:
            out = ref_attn.paged_attention_extend(q, kvc, 0, list(range(B)), lens, Hq)
            starts = list(lens)
        arrays[tag + "_q"] = q.float().numpy()
        arrays[tag + "_k"] = kvc._k.float().numpy()
        arrays[tag + "_v"] = kvc._v.float().numpy()
        arrays[tag + "_out"] = out.float().numpy()
        arrays[tag + "_starts"] = np.array(starts, dtype=np.int64)
        arrays[tag + "_tables"] = np.array([t + [-1] * (64 - len(t)) for t in kvc.block_tables], dtype=np.int64)
        arrays[tag + "_meta"] = np.array([Hq, Hkv, d, bs, chunk, cap], dtype=np.int64)

    attn_case("dec_f32_small", torch.float32, 4, 2, 8, 4, [8, 0, 6], 1, 11)
    attn_case("dec_f32_d64", torch.float32, 4, 2, 64, 16, [40, 3, 77, 16], 1, 12)
    attn_case("ext_f32_d64", torch.float32, 4, 2, 64, 16, [33, 0, 50], 5, 13)
    attn_case("dec_bf16_d128", torch.bfloat16, 12, 2, 128, 16, [300, 17, 129, 64], 1, 14)
    attn_case("ext_bf16_d128", torch.bfloat16, 12, 2, 128, 16, [256, 31, 100], 6, 15)
    attn_case("dec_bf16_d64_r7", torch.bfloat16, 14, 2, 64, 16, [200, 15, 48], 1, 16)
    g = torch.Generator().manual_seed(17)
    q = torch.randn(2, 6, 4, 8, generator=g)
    k = torch.randn(2, 6, 2, 8, generator=g)
    v = torch.randn(2, 6, 2, 8, generator=g)
    arrays["pre_f32_q"], arrays["pre_f32_k"], arrays["pre_f32_v"] = q.numpy(), k.numpy(), v.numpy()
    arrays["pre_f32_lens"] = np.array([4, 6])
    arrays["pre_f32_out"] = ref_attn.paged_attention_prefill_chunk(q, k, v, 4, [4, 6]).numpy()
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **arrays)

    # ---------------------------------------------------------- sampler
    samp = {"probs": [], "residual": [], "accept_kat": [], "accept_stoch": [], "draw": []}
    g = torch.Generator().manual_seed(21)
    for T, V in ((1.0, 64), (0.8, 400), (0.0, 50), (2.5, 7)):
        logits = torch.randn(3, V, generator=g) * 2.0
        p = ref_sampler.logits_to_probs(logits, SpecSampling(temperature=T))
        samp["probs"].append({"T": T, "logits": logits.tolist(), "probs": p.tolist()})
    for V in (16, 300):
        p = torch.softmax(torch.randn(V, generator=g), -1)
        qq = torch.softmax(torch.randn(V, generator=g), -1)
        samp["residual"].append({"p": p.tolist(), "q": qq.tolist(),
                                 "residual": ref_sampler.residual_distribution(p, qq).tolist()})
    u_rng = np.random.default_rng(99)
    for V in (5, 100, 4096):
        w = torch.softmax(torch.randn(V, generator=g) * 3, -1).numpy()
        us = u_rng.random(8, dtype=np.float32)
        samp["draw"].append({"w": w.tolist(), "u": us.tolist(), "idx": [sample_index(w, u) for u in us]})

    def one_hot(t, V=8):
        x = torch.zeros(V)
        x[t] = 1.0
        return x

    stream_vals = []

    def install_stream(values):
        it = iter([float(x) for x in values])
        ref_spec._draw_uniform = lambda gen: next(it)
        ref_spec.sample_token = lambda probs, gen=None: sample_index(probs.detach().float().numpy(), next(it))
        return it

    kat_cases = [
        ({0: torch.stack([one_hot(3)] * 3)}, {0: [one_hot(3)] * 2}, {0: [3, 3]}),
        ({0: torch.stack([one_hot(5), one_hot(5)])}, {0: [one_hot(2)]}, {0: [2]}),
        ({0: torch.stack([one_hot(1), one_hot(4), one_hot(4)])}, {0: [one_hot(1), one_hot(7)]}, {0: [1, 7]}),
    ]
    for p_by, q_by, prop in kat_cases:
        us = u_rng.random(16, dtype=np.float32)
        install_stream(us)
        acc = ref_spec.batch_accept(p_by, q_by, prop, None)
        samp["accept_kat"].append({"p": {k: v.tolist() for k, v in p_by.items()},
                                   "q": {k: [r.tolist() for r in v] for k, v in q_by.items()},
                                   "proposals": prop, "u": us.tolist(), "accepted": acc})
    for case in range(6):
        B, gamma, V = (3, 4, 50) if case < 3 else (5, 2, 400)
        temp = 1.0 if case % 2 == 0 else 0.6
        pl = torch.randn(B, gamma + 1, V, generator=g) * 2.0
        ql = pl[:, :gamma] + torch.randn(B, gamma, V, generator=g) * (0.3 + 0.4 * case)
        sc = SpecSampling(temperature=temp)
        p_by = {b: ref_sampler.logits_to_probs(pl[b], sc) for b in range(B)}
        q_by = {b: [ref_sampler.logits_to_probs(ql[b, j], sc) for j in range(gamma)] for b in range(B)}
        prop = {b: [int(torch.argmax(q_by[b][j]).item()) if (b + j) % 2 == 0 else int((b * 7 + j) % V)
                    for j in range(gamma)] for b in range(B)}
        us = u_rng.random(B * (gamma + 1), dtype=np.float32)
        install_stream(us)
        acc = ref_spec.batch_accept(p_by, q_by, prop, None)
        samp["accept_stoch"].append({"T": temp, "p_logits": pl.tolist(), "q_logits": ql.tolist(),
                                     "proposals": {str(k): v for k, v in prop.items()}, "u": us.tolist(),
                                     "accepted": {str(k): v for k, v in acc.items()}})
    with open(os.path.join(HERE, "sampler.json"), "w") as f:
        json.dump(samp, f)

    # ---------------------------------------------------------- C1 runs
    C1 = workloads.C1

    class IdTok:
        eos_token_id = None

        def encode(self, x):
            return list(x)

    def c1_model(name, seed):
        cfg = workloads.shape_config(name, rope_theta=1e6, max_position_embeddings=4096)
        torch.manual_seed(0)
        m = QwenPagedModel(cfg, torch.device("cpu"))
        state = {k: torch.from_numpy(v) for k, v in weights.qwen_numpy_state(cfg, seed, C1["weight_std"]).items()}
        missing, _ = m.load_state_dict(state, strict=False)
        assert not missing, missing
        m.tokenizer = IdTok()
        return m

    target = c1_model("c1-target", C1["target_seed"])
    draft = c1_model("c1-draft", C1["draft_seed"])
    reqs_raw = workloads.c1_requests(0)
    runs = {}
    for label, temp in (("greedy", 0.0), ("t1", 1.0)):
        us = workloads.c1_uniforms(0)
        it = install_stream(us)
        consumed = [0]

        def sched_sample(self, probs, generator, _it=it, _c=consumed):
            if self.sampling.is_greedy:
                return int(probs)
            _c[0] += 1
            return sample_index(probs.detach().float().numpy(), next(_it))

        ref_sched.PagedScheduler._sample = sched_sample
        cfg = EngineConfig(block_size=C1["block_size"], max_num_blocks=64)
        kv_t = ref_sched.build_kv(target, cfg, torch.device("cpu"))
        kv_d = ref_sched.build_kv(draft, cfg, torch.device("cpu"))
        sched = ref_spec.SpeculativePagedScheduler(target, kv_t, draft, kv_d, cfg, SpecSampling(temperature=temp),
                                                   C1["gamma"])
        snaps = []
        orig_step = ref_spec.SpeculativePagedScheduler._spec_step

        def step_and_snap(self, running, result, generator, _orig=orig_step, _snaps=snaps):
            _orig(self, running, result, generator)
            _snaps.append({"target": copy.deepcopy(self.kv.block_tables),
                           "target_len": list(self.kv.seq_lengths),
                           "draft": copy.deepcopy(self.draft_kv.block_tables),
                           "draft_len": list(self.draft_kv.seq_lengths)})

        ref_spec.SpeculativePagedScheduler._spec_step = step_and_snap
        reqs = [WorkloadRequest(prompt=ids, max_new_tokens=n, arrive_time=a) for ids, n, a in reqs_raw]
        with torch.no_grad():
            res = sched.run_spec_continuous(reqs, seed=0, measure=False)
        ref_spec.SpeculativePagedScheduler._spec_step = orig_step
        runs[label] = {
            "temperature": temp,
            "generated": [s.generated for s in res.sequences],
            "tokens_per_round": res.tokens_per_round,
            "steps": res.steps,
            "draft_forward_calls": res.draft_forward_calls,
            "kv_peak_blocks": res.kv_peak_blocks,
            "draft_kv_peak_blocks": res.draft_kv_peak_blocks,
            "snapshots": snaps,
        }
    with open(os.path.join(HERE, "c1_spec.json"), "w") as f:
        json.dump({"config": C1, "capacity": 64, "runs": runs}, f)

    # ---------------------------------------------------------- committed toy goldens
    ref_sched.PagedScheduler._sample = lambda self, probs, gen: int(probs)
    with open(os.path.join(args.reference, "results", "cpu", "spec_correctness_toy.json")) as f:
        spec_json = json.load(f)
    with open(os.path.join(args.reference, "results", "cpu", "engine_correctness_toy.json")) as f:
        eng_json = json.load(f)
    seed = spec_json["seed"]
    wl = WorkloadConfig(prompts=__import__("engine.config", fromlist=["x"]).DEFAULT_PROMPTS, num_requests=6,
                        min_tokens=4, max_tokens=16, arrival_window=4, seed=seed)
    requests = build_workload(wl, build_generator(seed))
    tgt = ToyPagedLM(ToyConfig(seed=seed, vocab_size=16), torch.device("cpu"))
    drf = ToyPagedLM(ToyConfig(seed=7, hidden_size=48, num_layers=2, num_attention_heads=4, num_key_value_heads=2,
                               head_dim=12, vocab_size=16), torch.device("cpu"))
    cfg = EngineConfig(block_size=16, max_num_blocks=256, max_batch=16)
    greedy = SpecSampling(temperature=0.0)
    sched = ref_spec.SpeculativePagedScheduler(tgt, ref_sched.build_kv(tgt, cfg, torch.device("cpu")), drf,
                                               ref_sched.build_kv(drf, cfg, torch.device("cpu")), cfg, greedy,
                                               spec_json["gamma"])
    spec = sched.run_spec_continuous(requests, seed=seed, measure=False)
    spec_rows = [r["spec_generated"] for r in spec_json["reports"][0]["rows"]]
    assert [s.generated for s in spec.sequences] == spec_rows, "reference does not reproduce its spec golden"

    eseed = 20260920
    wl = WorkloadConfig(prompts=ENGINE_PROMPTS, num_requests=6, min_tokens=4, max_tokens=16, arrival_window=4,
                        seed=eseed)
    erequests = build_workload(wl, build_generator(eseed))
    emodel = ToyPagedLM(ToyConfig(seed=eseed), torch.device("cpu"))
    ecfg = EngineConfig(block_size=16, max_num_blocks=512, max_batch=8)
    eres = ref_sched.PagedScheduler(emodel, ref_sched.build_kv(emodel, ecfg, torch.device("cpu")), ecfg,
                                    __import__("engine.config", fromlist=["x"]).SamplingConfig(temperature=0.0)
                                    ).run_continuous(erequests, seed=eseed, measure=False)
    eng_rows = [r["generated"] for r in eng_json["reports"][0]["rows"]]
    assert [s.generated for s in eres.sequences] == eng_rows, "reference does not reproduce its engine golden"
    with open(os.path.join(HERE, "toy_correctness.json"), "w") as f:
        json.dump({
            "spec": {"seed": seed, "gamma": spec_json["gamma"], "block_size": 16, "max_num_blocks": 256,
                     "requests": [r.__dict__ for r in requests], "generated": spec_rows,
                     "tokens_per_round": spec.tokens_per_round},
            "engine": {"seed": eseed, "block_size": 16, "max_num_blocks": 512,
                       "requests": [r.__dict__ for r in erequests], "generated": eng_rows},
        }, f)
    print("golden fixtures written to", HERE)
    return 0


if __name__ == "__main__":
    sys.exit(main())
