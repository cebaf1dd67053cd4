"""Benchmark of the paged-KV hot path on B200 (one JSON line on stdout).

Workload (default, BASELINE.json configs[1] = "C2"): paged decode attention
plus KV append with Qwen2.5-1.5B attention shapes -- 28 layers, 12 q heads,
2 KV heads, head_dim 128, block_size 16, bf16, batch 64 per GPU, context
lengths U[512, 4096] (seeded), block tables a random permutation of a pool
that holds every context, Q/K/V ~ N(0, 1).  One *step* = every sequence
appends one token (K/V of all 28 layers) and attends its context + itself in
every layer; the sequences are then rewound by one position so every step
sees the same C2 context distribution.  tokens/s = batch * steps / time.

Arms:
  (default)          the B200 kernels: the timed region replays one CUDA
                     graph per step (28 x [append + paged attention]) after a
                     reserve launch, and a release launch after it; inputs
                     resident in HBM.  ``e2e`` re-measures through the public
                     per-layer API with pinned-host inputs copied in and the
                     attention outputs copied back every step.
  --impl reference   the reference's CPU algorithm (the numpy oracle port, all
                     host threads) on a bounded sample of the same workload.

``--workload c3`` instead times the verify step of
a speculative round at gamma = 5: 32 sequences per GPU with contexts
U[256, 2048] reserve gamma+1 positions, every one of the 28 layers appends
their K/V and runs the (gamma+1)-row extend attention (Qwen2.5-1.5B
attention shapes, bf16), then target and draft logits ~ N(0, 2) (fp32,
vocab 151936, fixed draft proposals drawn from the draft distribution) go
through temperature-1 softmax and the fused rejection sampler with fp32
uniforms from a seeded stream, and the commit kernel rewinds every block
table to its accept length.  tokens/s = committed tokens / time.

``--workload c5`` times the attention of one
long-context round at gamma = 6 per GPU: 16 sequences with contexts
U[8192, 32768] run 6 draft decode steps over 28 layers of the Qwen2.5-1.5B
attention shape, then the 7-row verify over 36 layers of the 3B shape
(16 q heads), each layer one fused append + attention launch; tokens/s =
batch * 7 verified positions per round / round time, with the verify and
the decode rooflines reported separately.

Multi-GPU (torchrun): every rank runs its own batch of sequences (weak
scaling, no data-path collective); a barrier brackets the timed region and the
slowest rank's time is used.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "speculative-decoding-lab_b200")
for _p in (PKG, ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "spec-decode tokens/s (paged KV, 1/2/4/8 GPU); paged-attn HBM GB/s vs 8 TB/s"
C2 = dict(layers=28, q_heads=12, kv_heads=2, head_dim=128, block_size=16, batch=64, ctx_lo=512, ctx_hi=4096)
# DRAM bytes (read + write) of one C2 attention launch of attn_tc_kernel, from the
# ncu --set full capture summarised under profiles/ (refreshed when re-profiled).
C2_ATTN_TRAFFIC = 154_167_040 + 3_741_184
# DRAM bytes per algorithmic byte of C4's two attention main kernels under the
# ragged plan, from ncu --set full captures at 358 sequences (summaries under
# profiles/): the bench's rooflines run at the run's heaviest round, whose size
# varies, so traffic is scaled by the algorithmic bytes the launch moves
C4_DECODE_TRAFFIC_RATIO = (135_227_136 + 4_350_464) / 134_700_000
C4_VERIFY_TRAFFIC_RATIO = (276_881_152 + 14_143_232) / 282_200_000

# kernel names of the attention op per attention_kernel() answer
ATTN_KERNELS = {
    "mma": "attn_tc_kernel (+ attn_combine_kernel when split)",
    "mma_rows": "attn_rows_kernel (+ attn_combine_kernel when split)",
    "mma_direct": "attn_direct_kernel (+ attn_combine_kernel when split)",
    "tcgen05": "attn_sk_kernel + attn_sk_combine_kernel (persistent tcgen05)",
    "generic": "attn_generic_kernel",
}
C3 = dict(layers=28, q_heads=12, kv_heads=2, head_dim=128, block_size=16, batch=32, ctx_lo=256, ctx_hi=2048,
          gamma=5, vocab=151936, temperature=1.0, logit_std=2.0)
# C5: Qwen2.5-3B-shaped target, 1.5B-shaped draft, 16 sequences per GPU
C5 = dict(target_layers=36, target_q_heads=16, draft_layers=28, draft_q_heads=12, kv_heads=2, head_dim=128,
          block_size=16, batch=16, ctx_lo=8192, ctx_hi=32768, gamma=6)


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.3)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU baseline
class CpuC2:
    """The reference algorithm (numpy oracle port) on a bounded sample of C2.

    A unit is one (sequence, layer) pair: write the new token's K/V into the
    paged pool, gather the sequence's pages and attend context + itself (the
    per-sequence loop of engine/attention.py:96-118 after engine/kv.py:125-147).
    Units run on layer 0 of the 64 sequences, threaded over sequences, for a
    fixed wall-clock budget; tokens/s = 64 / (64 * 28 * seconds-per-unit).
    """

    def __init__(self, seed: int = 0, threads: int = 0) -> None:
        from engine.workloads import c2_layout
        from oracle import kv as okv

        c = C2
        self.ctx, tables, cap = c2_layout(seed, c["batch"], c["ctx_lo"], c["ctx_hi"], c["block_size"])
        rng = np.random.default_rng(seed)
        self.kv = okv.PagedKVCache(1, c["kv_heads"], c["head_dim"], cap, c["block_size"])
        self.kv.k[:] = rng.standard_normal(self.kv.k.shape, dtype=np.float32)
        self.kv.v[:] = rng.standard_normal(self.kv.v.shape, dtype=np.float32)
        for sid, t in enumerate(tables):
            self.kv.add_sequence(sid)
            self.kv.block_tables[sid] = list(t)
            self.kv.seq_lengths[sid] = self.ctx[sid]
        self.q = rng.standard_normal((c["batch"], c["q_heads"], c["head_dim"])).astype(np.float32)
        self.knew = rng.standard_normal((c["batch"], c["kv_heads"], c["head_dim"])).astype(np.float32)
        self.threads = threads or (os.cpu_count() or 1)

    def _unit(self, b: int) -> int:
        from oracle import attention as oatt

        ctx = self.ctx[b]
        self.kv.write(0, b, ctx, self.knew[b], self.knew[b])
        k, v = self.kv.gather(0, b, ctx + 1)
        oatt.attend(self.q[b][None], k, v, [ctx + 1])
        self.kv.seq_lengths[b] = ctx
        return 1

    def measure(self, seconds: float):
        from concurrent.futures import ThreadPoolExecutor

        c = C2
        done = 0
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=self.threads) as ex:
            while True:
                done += sum(ex.map(self._unit, range(c["batch"])))
                if time.perf_counter() - t0 >= seconds:
                    break
        dt = time.perf_counter() - t0
        step_s = c["batch"] * c["layers"] * dt / done
        return {
            "value": round(c["batch"] / step_s, 4),
            "unit": "tokens/s",
            "cores": self.threads,
            "kind": "port",
            "sample": "{} (sequence, layer) units of C2 (layer 0 of the 64 sequences: KV write + paged decode "
                      "attention, numpy fp64) in {:.2f} s on {} threads, scaled to 28 layers x 64 sequences "
                      "per step".format(done, dt, self.threads),
        }


class CpuC3:
    """The reference algorithm (numpy oracle port) on a bounded sample of C3.

    A unit is one sequence's verify step: for every layer write the gamma+1
    new K/V rows into the paged pool and run the masked extend attention
    (engine/attention.py:170-215 after engine/kv.py:125-147); then softmax the
    sequence's 2*gamma+1 logit rows, run batch_accept
    (engine/spec_scheduler.py:46-88) and truncate the table to the accept
    length (engine/kv.py:150-162).  Units run on ``layers_sampled`` layers
    and are scaled to 28; tokens/s = committed tokens / scaled seconds.
    """

    def __init__(self, seed: int = 0, threads: int = 0, layers_sampled: int = 2, batch: int = 32) -> None:
        from engine.workloads import c2_layout
        from oracle import kv as okv
        from oracle import sampler as osm

        c = C3
        self.gamma = c["gamma"]
        self.chunk = c["gamma"] + 1
        self.layers = layers_sampled
        self.B = batch
        bs = c["block_size"]
        self.ctx, _, _ = c2_layout(seed, batch, c["ctx_lo"], c["ctx_hi"], bs)
        cap = sum(-(-(x + self.chunk) // bs) for x in self.ctx) + batch
        rng = np.random.default_rng(seed)
        self.kv = okv.PagedKVCache(layers_sampled, c["kv_heads"], c["head_dim"], cap, bs)
        self.kv.k[:] = rng.standard_normal(self.kv.k.shape, dtype=np.float32)
        self.kv.v[:] = rng.standard_normal(self.kv.v.shape, dtype=np.float32)
        for sid, n in enumerate(self.ctx):
            self.kv.add_sequence(sid)
            self.kv.reserve([sid], [0], [n])
        self.lock = threading.Lock()  # the pool's free list is shared by the worker threads
        H, d, V = c["q_heads"], c["head_dim"], c["vocab"]
        self.q = rng.standard_normal((batch, self.chunk, H, d)).astype(np.float32)
        self.knew = rng.standard_normal((batch, self.chunk, c["kv_heads"], d)).astype(np.float32)
        self.p_logits = (rng.standard_normal((batch, self.chunk, V)) * c["logit_std"]).astype(np.float32)
        self.q_logits = (rng.standard_normal((batch, self.gamma, V)) * c["logit_std"]).astype(np.float32)
        self.uniforms = rng.random(1 << 16, dtype=np.float32)
        self.props = []
        for b in range(batch):
            qp = osm.logits_to_probs(self.q_logits[b], c["temperature"])
            self.props.append([osm.sample_index(qp[t], self.uniforms[b * self.gamma + t]) for t in range(self.gamma)])
        self.threads = threads or (os.cpu_count() or 1)

    def _unit(self, b: int) -> int:
        from oracle import attention as oatt
        from oracle import sampler as osm

        c = C3
        start = self.ctx[b]
        t0 = time.perf_counter()
        with self.lock:
            slots = self.kv.reserve([b], [start], [self.chunk])
        for layer in range(self.layers):
            self.kv.append(layer, slots, self.knew[b], self.knew[b])
            oatt.paged_attention_extend(self.q[b][None], self.kv, layer, [b], [start])
        t1 = time.perf_counter()
        p = osm.logits_to_probs(self.p_logits[b], c["temperature"])
        q = osm.logits_to_probs(self.q_logits[b], c["temperature"])
        stream = osm.UniformStream(self.uniforms[(b * 97) % 4096:])
        acc = osm.batch_accept([p], [list(q)], [self.props[b]], stream)[0]
        with self.lock:
            self.kv.truncate(b, start + len(acc))
        return len(acc), t1 - t0, time.perf_counter() - t1

    def measure(self, seconds: float):
        from concurrent.futures import ThreadPoolExecutor

        c = C3
        toks = units = 0
        t_attn = t_samp = 0.0
        t0 = time.perf_counter()
        with ThreadPoolExecutor(max_workers=self.threads) as ex:
            while True:
                res = list(ex.map(self._unit, range(self.B)))
                toks += sum(r[0] for r in res)
                t_attn += sum(r[1] for r in res)
                t_samp += sum(r[2] for r in res)
                units += len(res)
                if time.perf_counter() - t0 >= seconds:
                    break
        dt = time.perf_counter() - t0
        # scale the per-layer share of the wall time from the sampled layers to all 28
        f = t_attn / max(t_attn + t_samp, 1e-12)
        scaled = dt * (f * c["layers"] / self.layers + (1.0 - f))
        return {
            "value": round(toks / scaled, 4),
            "unit": "tokens/s",
            "cores": self.threads,
            "kind": "port",
            "sample": "{} verify units of C3 ({} of 28 layers: K/V write + masked extend attention, then softmax "
                      "of 11 vocab rows, batch_accept and truncate; numpy) in {:.2f} s on {} threads, {} committed "
                      "tokens; the per-layer share ({:.0%}) of the time scaled by 28/{}".format(
                          units, self.layers, dt, self.threads, toks, f, self.layers),
        }


class _Budget(Exception):
    pass


class CpuC4:
    """The reference algorithm (numpy oracle port) on a bounded sample of C4.

    The oracle's speculative scheduler (engine/spec_scheduler.py:110-322
    restated: prefill on admission, gamma draft decodes, the gamma+1-row
    verify, batch_accept, rewind / catch-up / clear) serves the first
    ``batch`` requests of the C4 stream, all admitted at once, with both
    models cut to one decoder layer (Qwen2.5-1.5B and 0.5B shapes, full
    151,936-row vocab heads, weights N(0, 0.02), embeddings tied to the
    heads to halve host memory) until ``seconds`` of host time are spent.  The time inside
    the decoder layers is scaled to the full depth (28 and 24 layers).
    Prefill is charged per request in proportion to the share of its output
    the sample produced: tokens/s = tokens / (round time + prefill time x
    tokens / requested tokens).
    """

    def __init__(self, seed: int = 0, threads: int = 0, batch: int = 8) -> None:
        from engine import workloads
        from engine.weights import qwen_numpy_state
        from oracle.model import NumpyPagedLM, rotary_table

        assert 151936 % 128 == 0

        c = workloads.C4
        self.c = c
        self.batch = batch
        self.threads = threads or (os.cpu_count() or 1)
        self.models = []
        self.depth = []
        for name, s in ((c["target"], 1), (c["draft"], 2)):
            full = workloads.shape_config(name)
            cfg = workloads.shape_config(name, num_hidden_layers=1, tie_word_embeddings=True)
            # the vocab rows repeat one random block of 1187 rows (151936 = 128 x 1187): the same
            # arithmetic as distinct rows, without drawing 10^8 normals per model
            V, H = cfg.vocab_size, cfg.hidden_size
            cfg_small = workloads.shape_config(name, num_hidden_layers=1, tie_word_embeddings=True,
                                               vocab_size=V // 128)
            st = qwen_numpy_state(cfg_small, seed * 2 + s, 0.02)
            st["embed_tokens.weight"] = np.tile(st["embed_tokens.weight"], (128, 1))
            st["lm_head.weight"] = st["embed_tokens.weight"]
            rope = rotary_table(cfg.head_dim, cfg.rope_theta, c["prompt_cap"] + c["out_hi"] + 16)
            m = NumpyPagedLM(st, 1, cfg.num_attention_heads, cfg.num_key_value_heads, cfg.head_dim, rope, "qwen")
            self.models.append(m)
            self.depth.append(int(full.num_hidden_layers))
        self.reqs = workloads.c4_requests(seed, batch, 1.0, c["vocab"])

    def measure(self, seconds: float):
        from oracle import kv as okv
        from oracle import sampler as osm
        from oracle import scheduler as osched

        c = self.c
        acc = {"layers": [0.0, 0.0], "prefill": 0.0, "prefill_layers": [0.0, 0.0]}
        state = {"in_prefill": False}
        for i, m in enumerate(self.models):
            layer_fn = type(m)._layer
            prefill_fn = type(m).prefill

            def timed_layer(*a, _f=layer_fn, _m=m, _i=i, **k):
                t = time.perf_counter()
                try:
                    return _f(_m, *a, **k)
                finally:
                    key = "prefill_layers" if state["in_prefill"] else "layers"
                    acc[key][_i] += time.perf_counter() - t

            def timed_prefill(*a, _f=prefill_fn, _m=m, **k):
                t = time.perf_counter()
                state["in_prefill"] = True
                try:
                    return _f(_m, *a, **k)
                finally:
                    state["in_prefill"] = False
                    acc["prefill"] += time.perf_counter() - t

            m._layer = timed_layer
            m.prefill = timed_prefill
        tgt, dft = self.models
        cap_t = sum(-(-(len(ids) + new + 16) // 16) for ids, new, _ in self.reqs) + 8
        kv_t = okv.PagedKVCache(1, tgt.nkv, tgt.d, cap_t, 16)
        kv_d = okv.PagedKVCache(1, dft.nkv, dft.d, cap_t, 16)
        us = np.random.default_rng(12345).random(1 << 20, dtype=np.float32)
        reqs = [osched.Req(list(ids), new, 0) for ids, new, _ in self.reqs]
        res = osched.RunResult()
        t0 = time.perf_counter()

        def hook():
            if time.perf_counter() - t0 >= seconds:
                raise _Budget()

        try:
            osched.run_spec_continuous(tgt, kv_t, dft, kv_d, reqs, c["gamma"], c["temperature"],
                                       stream=osm.UniformStream(us), round_hook=hook, result=res)
        except _Budget:
            pass
        wall = time.perf_counter() - t0
        tokens = sum(len(s.generated) for s in res.sequences)
        requested = sum(s.max_new_tokens for s in res.sequences)
        rounds = len(res.tokens_per_round) // max(1, len(res.sequences))
        lt, ld = acc["layers"]
        plt, pld = acc["prefill_layers"]
        scale_t, scale_d = self.depth[0], self.depth[1]
        prefill_scaled = acc["prefill"] + plt * (scale_t - 1) + pld * (scale_d - 1)
        round_wall = wall - acc["prefill"]
        round_scaled = round_wall + lt * (scale_t - 1) + ld * (scale_d - 1)
        charged = round_scaled + prefill_scaled * tokens / max(1, requested)
        value = tokens / charged
        return {
            "value": round(value, 4),
            "unit": "tokens/s",
            "cores": self.threads,
            "kind": "port",
            "sample": "oracle speculative scheduler (numpy: fp32 GEMMs on {} BLAS threads, fp64 attention) "
                      "serving the first {} C4 requests with both models cut to 1 decoder layer: {:.2f} s of "
                      "host time ({:.2f} s prefill, ~{} rounds), {} tokens of {} requested; decoder-layer time "
                      "scaled to 28 / 24 layers and prefill charged in proportion to the output produced, "
                      "{:.1f} s charged".format(self.threads, len(res.sequences), wall, acc["prefill"], rounds,
                                               tokens, requested, charged),
            "sample_seconds": round(wall, 3),
        }


# --------------------------------------------------------------- GPU arm
def run_gpu(args, rank: int, world: int, device):
    import torch

    from engine import _lib
    from engine.attention import AttnBatch, attention_kernel, attention_launches, paged_attention
    from engine.kv import PagedKVCache
    from engine.workloads import c2_layout

    c = dict(C2)
    akw = dict(use_umma=UMMA_FLAG[args.attn_kernel], mma_layout=LAYOUT_FLAG[args.mma_layout],
               overlap_layers=_overlap_layers(args))
    fused = args.append == "fused"
    L = args.layers
    B = args.batch
    Hq, Hkv, d, bs = c["q_heads"], c["kv_heads"], c["head_dim"], c["block_size"]
    seed = args.seed + rank
    ctx, _, _ = c2_layout(seed, B, c["ctx_lo"], c["ctx_hi"], bs)
    cap = sum(-(-(x + 1) // bs) for x in ctx) + B
    kv = PagedKVCache(L, Hkv, d, cap, bs, device, torch.bfloat16, max_blocks_per_seq=-(-(c["ctx_hi"] + 2) // bs),
                      max_seqs=B)
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    kv.allocator._free_stack.copy_(torch.randperm(cap, generator=g).to(torch.int32))  # random-permutation pool
    sids = list(range(B))
    for sid in sids:
        kv.add_sequence(sid)
    kv.reserve(sids, [0] * B, ctx)
    gd = torch.Generator(device=device)
    gd.manual_seed(seed)
    kv._k.normal_(generator=gd)
    kv._v.normal_(generator=gd)
    q = torch.randn((L, B, 1, Hq, d), generator=gd, device=device, dtype=torch.float32).to(torch.bfloat16)
    knew = torch.randn((L, B, Hkv, d), generator=gd, device=device, dtype=torch.float32).to(torch.bfloat16)
    vnew = torch.randn((L, B, Hkv, d), generator=gd, device=device, dtype=torch.float32).to(torch.bfloat16)
    out = torch.empty((L, B, 1, Hq, d), device=device, dtype=torch.bfloat16)
    batch = AttnBatch.from_lists(device, sids, ctx, 1)  # new token at position ctx attends [0, ctx]
    slots_static = torch.empty(B, dtype=torch.int32, device=device)
    rel_flags = [_lib.REL_TRUNCATE] * B
    stream = torch.cuda.current_stream(device)

    def step_layers(with_append=True):
        for layer in range(L):
            if with_append and fused:  # store the new K/V row inside the attention launch
                paged_attention(q[layer], kv, layer, batch, out=out[layer], **akw, k_new=knew[layer],
                                v_new=vnew[layer])
                continue
            if with_append:
                kv.append(layer, slots_static, knew[layer], vnew[layer])
            paged_attention(q[layer], kv, layer, batch, out=out[layer], **akw)

    # warm up every code path once outside capture (attributes, workspace)
    slots_static.copy_(kv.reserve(sids, ctx, [1] * B))
    step_layers()
    kv.release(sids, ctx, rel_flags)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):  # captured on torch's side stream, replayed on `stream`
        step_layers()
    attn_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(attn_graph):  # the attention op as the step launches it
        step_layers(with_append=fused)
    torch.cuda.synchronize(device)

    def device_step():
        slots_static.copy_(kv.reserve(sids, ctx, [1] * B))
        graph.replay()
        kv.release(sids, ctx, rel_flags)

    for _ in range(args.warmup):
        device_step()
    torch.cuda.synchronize(device)
    kv.check_errors()
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    clocks = ClockSampler(device.index if device.index is not None else 0) if rank == 0 else None
    if clocks:
        clocks.start()
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        device_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    step_ms = e0.elapsed_time(e1) / args.steps

    # roofline: the attention op alone (main kernel + split combine), 28 launches per replay
    reps = max(3, args.steps // 4)
    slots_static.copy_(kv.reserve(sids, ctx, [1] * B))  # back position ctx while attention reads it
    for _ in range(2):
        attn_graph.replay()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(reps):
        attn_graph.replay()
    a1.record(stream)
    torch.cuda.synchronize(device)
    kv.release(sids, ctx, rel_flags)
    attn_ms = a0.elapsed_time(a1) / (reps * L)
    clk = clocks.stop() if clocks else None
    kv.check_errors()

    # e2e through the public per-layer API with pinned host buffers
    q_h = q.cpu().pin_memory()
    k_h = knew.cpu().pin_memory()
    v_h = vnew.cpu().pin_memory()
    o_h = torch.empty(out.shape, dtype=out.dtype).pin_memory()
    h2d = q_h.numel() * 2 + k_h.numel() * 2 + v_h.numel() * 2
    d2h = o_h.numel() * 2

    # Copies run on their own stream, pipelined with the layers: step s+1's
    # inputs go up while step s computes, and step s's outputs come down
    # while step s+1 computes (two device buffer sets, ordered by events).
    comp = torch.cuda.current_stream(device)
    copy_stream = torch.cuda.Stream(device)
    bufs = [(torch.empty_like(q), torch.empty_like(knew), torch.empty_like(vnew), torch.empty_like(out))
            for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    out_ready = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]

    e2e_akw = dict(akw, overlap_layers=False)

    def upload(i):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(freed[i])  # step s-2 has read buffer set i and its outputs are down
            qd, kd, vd, _ = bufs[i]
            qd.copy_(q_h, non_blocking=True)
            kd.copy_(k_h, non_blocking=True)
            vd.copy_(v_h, non_blocking=True)
            in_ready[i].record(copy_stream)

    def e2e_step(i):
        qd, kd, vd, od = bufs[i]
        comp.wait_event(in_ready[i])
        slots = kv.reserve(sids, ctx, [1] * B)
        b2 = AttnBatch.from_lists(device, sids, ctx, 1)
        for layer in range(L):
            # eager calls: the host paces the launches, so layers do not overlap
            if fused:
                paged_attention(qd[layer], kv, layer, b2, out=od[layer], **e2e_akw, k_new=kd[layer],
                                v_new=vd[layer])
            else:
                kv.append(layer, slots, kd[layer], vd[layer])
                paged_attention(qd[layer], kv, layer, b2, out=od[layer], **e2e_akw)
        kv.release(sids, ctx, rel_flags)
        out_ready[i].record(comp)
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(out_ready[i])
            o_h.copy_(od, non_blocking=True)
            freed[i].record(copy_stream)

    def e2e_run(n):
        upload(0)
        for st in range(n):
            if st + 1 < n:
                upload((st + 1) % 2)
            e2e_step(st % 2)

    e2e_steps = max(3, args.steps // 4)
    e2e_run(max(1, args.warmup))
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    e2e_run(e2e_steps)
    torch.cuda.synchronize(device)
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / e2e_steps
    kv.check_errors()
    # parity spot-check: the public-API outputs equal the graph path's, bit for bit
    device_step()
    torch.cuda.synchronize(device)
    if not torch.equal(o_h.to(device), out):
        raise RuntimeError("e2e outputs differ from the graph path")

    attn_bytes = sum((x + 1) * 2 * Hkv * d * 2 for x in ctx) + 2 * B * Hq * d * 2 + sum(-(-(x + 1) // bs) * 4 for x in ctx)
    if fused:  # the op also reads the new K/V rows and writes them into their pages
        attn_bytes += 2 * (B * 2 * Hkv * d * 2)
        per_layer = attention_launches(q[0], kv, batch, **akw, k_new=knew[0], v_new=vnew[0])
    else:
        per_layer = 1 + attention_launches(q[0], kv, batch, **akw)  # append + attention (+ merge)
    launches_per_step = 2 + L * per_layer  # + reserve + release
    if world > 1:
        t = torch.tensor([step_ms, e2e_ms, attn_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, e2e_ms, attn_ms = t.tolist()
    del graph, attn_graph
    kern = attention_kernel(q[0], kv, batch, **akw)
    return dict(kernel=kern, step_ms=step_ms, e2e_ms=e2e_ms, attn_ms=attn_ms, attn_bytes=attn_bytes, clocks=clk, h2d=h2d,
                d2h=d2h, launches=launches_per_step * args.steps, ctx_mean=float(np.mean(ctx)))


def run_gpu_c3(args, rank: int, world: int, device):
    """The C3 verify step (see the module docstring) on one GPU."""
    import ctypes

    import torch

    from engine import _lib
    from engine.attention import AttnBatch, attention_kernel, attention_launches, paged_attention
    from engine.kv import PagedKVCache
    from engine.workloads import c2_layout
    from specdec.sampler import UniformStream, probs_rows, sample_rows, spec_sample_logits

    c = dict(C3)
    akw = dict(use_umma=UMMA_FLAG[args.attn_kernel], mma_layout=LAYOUT_FLAG[args.mma_layout],
               overlap_layers=_overlap_layers(args))
    fused = args.append == "fused"
    L, B, gam = args.layers, args.batch, c["gamma"]
    chunk = gam + 1
    Hq, Hkv, d, bs, V, T = c["q_heads"], c["kv_heads"], c["head_dim"], c["block_size"], c["vocab"], c["temperature"]
    seed = args.seed + rank
    ctx, _, _ = c2_layout(seed, B, c["ctx_lo"], c["ctx_hi"], bs)
    cap = sum(-(-(x + chunk) // bs) for x in ctx) + B
    kv = PagedKVCache(L, Hkv, d, cap, bs, device, torch.bfloat16,
                      max_blocks_per_seq=-(-(c["ctx_hi"] + chunk + 1) // bs), max_seqs=B)
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    kv.allocator._free_stack.copy_(torch.randperm(cap, generator=g).to(torch.int32))  # random-permutation pool
    sids = list(range(B))
    for sid in sids:
        kv.add_sequence(sid)
    kv.reserve(sids, [0] * B, ctx)
    gd = torch.Generator(device=device)
    gd.manual_seed(seed)
    kv._k.normal_(generator=gd)
    kv._v.normal_(generator=gd)
    q = torch.randn((L, B, chunk, Hq, d), generator=gd, device=device).to(torch.bfloat16)
    knew = torch.randn((L, B * chunk, Hkv, d), generator=gd, device=device).to(torch.bfloat16)
    vnew = torch.randn((L, B * chunk, Hkv, d), generator=gd, device=device).to(torch.bfloat16)
    out = torch.empty((L, B, chunk, Hq, d), device=device, dtype=torch.bfloat16)
    p_logits = torch.randn((B, chunk, V), generator=gd, device=device) * c["logit_std"]
    q_logits = torch.randn((B, gam, V), generator=gd, device=device) * c["logit_std"]
    # the draft's proposals: its own draws from q, fixed for every step
    q_probs = probs_rows(q_logits, T, False)
    proposals = sample_rows(q_probs, UniformStream(device, seed=seed + 7)).view(B, gam)
    del q_probs
    ustream = UniformStream(device, seed=seed + 11)
    batch = AttnBatch.from_lists(device, sids, ctx, chunk)  # row j sits at ctx + j
    slots_static = torch.empty(B * chunk, dtype=torch.int32, device=device)
    tokens = torch.empty((B, chunk), dtype=torch.int32, device=device)
    n_out = torch.empty(B, dtype=torch.int32, device=device)
    packed = _lib.i32(sids + [1 << 30] * B + ctx, device)  # rows, remaining budget, round starts
    outs = torch.empty((3, B), dtype=torch.int32, device=device)
    lib = _lib.load()
    meta = ctypes.byref(kv.meta)

    def verify_layers(with_append=True):
        for layer in range(L):
            if with_append and fused:  # store the round's K/V rows inside the attention launch
                paged_attention(q[layer], kv, layer, batch, out=out[layer], **akw, k_new=knew[layer],
                                v_new=vnew[layer])
                continue
            if with_append:
                kv.append(layer, slots_static, knew[layer], vnew[layer])
            paged_attention(q[layer], kv, layer, batch, out=out[layer], **akw)

    def sample_commit():
        spec_sample_logits(p_logits, q_logits, T, proposals, ustream, err=kv.err_word, out=(tokens, n_out))
        _lib.check(lib.sdl_spec_commit(meta, None, B, packed.data_ptr(), n_out.data_ptr(), tokens.data_ptr(), chunk,
                                       packed.data_ptr() + 4 * B, -1, packed.data_ptr() + 8 * B, outs[0].data_ptr(),
                                       outs[1].data_ptr(), outs[2].data_ptr(), _lib.stream_handle(device)),
                   "sdl_spec_commit")

    # warm every path once outside capture
    slots_static.copy_(kv.reserve(sids, ctx, [chunk] * B))
    verify_layers()
    sample_commit()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        verify_layers()
    attn_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(attn_graph):  # the attention op as the step launches it
        verify_layers(with_append=fused)
    torch.cuda.synchronize(device)

    k_hist = torch.zeros((args.steps, B), dtype=torch.int32, device=device)

    def device_step(i=None):
        # the commit left every table at ctx + k; reserving from ctx backs the round's gamma+1 positions again
        slots_static.copy_(kv.reserve(sids, ctx, [chunk] * B))
        graph.replay()
        sample_commit()
        if i is not None:
            k_hist[i].copy_(outs[0])

    for _ in range(args.warmup):
        device_step()
    torch.cuda.synchronize(device)
    kv.resync()
    kv.check_errors()
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    clocks = ClockSampler(device.index if device.index is not None else 0) if rank == 0 else None
    if clocks:
        clocks.start()
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(torch.cuda.current_stream(device))
    for i in range(args.steps):
        device_step(i)
    e1.record(torch.cuda.current_stream(device))
    torch.cuda.synchronize(device)
    step_ms = e0.elapsed_time(e1) / args.steps
    committed = int(k_hist.sum().item())
    kv.resync()

    # roofline: the verify attention op alone, replayed over the 28 layers
    reps = max(3, args.steps // 4)
    slots_static.copy_(kv.reserve(sids, ctx, [chunk] * B))
    stream = torch.cuda.current_stream(device)
    for _ in range(2):
        attn_graph.replay()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(stream)
    for _ in range(reps):
        attn_graph.replay()
    a1.record(stream)
    torch.cuda.synchronize(device)
    attn_ms = a0.elapsed_time(a1) / (reps * L)
    # the fused sampler alone (statistics, accept walk, draw sums, draw)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(reps):
        spec_sample_logits(p_logits, q_logits, T, proposals, ustream, err=kv.err_word, out=(tokens, n_out))
    s1.record(stream)
    torch.cuda.synchronize(device)
    samp_ms = s0.elapsed_time(s1) / reps
    clk = clocks.stop() if clocks else None
    kv.release(sids, ctx, [_lib.REL_TRUNCATE] * B)
    kv.check_errors()

    # e2e through the public API: pinned host Q/K/V and logits in, tokens and accept lengths out
    q_h = q.cpu().pin_memory()
    k_h = knew.cpu().pin_memory()
    v_h = vnew.cpu().pin_memory()
    pl_h = p_logits.cpu().pin_memory()
    ql_h = q_logits.cpu().pin_memory()
    pr_h = proposals.cpu().pin_memory()
    tok_h = torch.empty((args.steps, B, chunk), dtype=torch.int32).pin_memory()
    k_out_h = torch.empty((args.steps, B), dtype=torch.int32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (q_h, k_h, v_h, pl_h, ql_h, pr_h))
    d2h = B * chunk * 4 + B * 4

    # Inputs go up on a copy stream, pipelined with the compute: step s+1's
    # Q/K/V, logits and proposals upload while step s runs (two device buffer
    # sets, ordered by events); tokens and accept lengths come back per step.
    comp = torch.cuda.current_stream(device)
    copy_stream = torch.cuda.Stream(device)
    hosts = (q_h, k_h, v_h, pl_h, ql_h, pr_h)
    ins = [tuple(torch.empty(t.shape, dtype=t.dtype, device=device) for t in hosts) for _ in range(2)]
    in_ready = [torch.cuda.Event() for _ in range(2)]
    freed = [torch.cuda.Event() for _ in range(2)]

    def upload(i):
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(freed[i])  # step s-2 has consumed buffer set i
            for dst, src in zip(ins[i], hosts):
                dst.copy_(src, non_blocking=True)
            in_ready[i].record(copy_stream)

    def e2e_step(st, i):
        qd, kd, vd, pld, qld, prd = ins[st % 2]
        comp.wait_event(in_ready[st % 2])
        slots = kv.reserve(sids, ctx, [chunk] * B)
        b2 = AttnBatch.from_lists(device, sids, ctx, chunk)
        od = torch.empty_like(out)
        for layer in range(L):
            if fused:
                paged_attention(qd[layer], kv, layer, b2, out=od[layer], **akw, k_new=kd[layer],
                                v_new=vd[layer])
            else:
                kv.append(layer, slots, kd[layer], vd[layer])
                paged_attention(qd[layer], kv, layer, b2, out=od[layer], **akw)
        toks, no = spec_sample_logits(pld, qld, T, prd, ustream, err=kv.err_word)
        _lib.check(lib.sdl_spec_commit(meta, None, B, packed.data_ptr(), no.data_ptr(), toks.data_ptr(), chunk,
                                       packed.data_ptr() + 4 * B, -1, packed.data_ptr() + 8 * B, outs[0].data_ptr(),
                                       outs[1].data_ptr(), outs[2].data_ptr(), _lib.stream_handle(device)),
                   "sdl_spec_commit")
        freed[st % 2].record(comp)
        tok_h[i].copy_(toks, non_blocking=True)
        k_out_h[i].copy_(outs[0], non_blocking=True)

    def e2e_run(n, record):
        upload(0)
        for st in range(n):
            if st + 1 < n:
                upload((st + 1) % 2)
            e2e_step(st, st if record else 0)

    e2e_steps = max(3, min(args.steps, 50))
    e2e_run(max(1, args.warmup), False)
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    e2e_run(e2e_steps, True)
    torch.cuda.synchronize(device)
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / e2e_steps
    e2e_committed = int(k_out_h[:e2e_steps].sum())
    kv.resync()
    kv.release(sids, ctx, [_lib.REL_TRUNCATE] * B)
    kv.check_errors()

    attn_bytes = (sum((x + chunk) * 2 * Hkv * d * 2 for x in ctx) + 2 * B * chunk * Hq * d * 2
                  + sum(-(-(x + chunk) // bs) * 4 for x in ctx))
    samp_bytes = B * (2 * gam + 1) * V * 4  # the fp32 logit rows of p and q, each read once
    launches_sampler = 4  # statistics, accept walk, draw sums, draw
    if fused:  # the op also reads the new K/V rows and writes them into their pages
        attn_bytes += 2 * (B * chunk * 2 * Hkv * d * 2)
        per_layer = attention_launches(q[0], kv, batch, **akw, k_new=knew[0], v_new=vnew[0])
    else:
        per_layer = 1 + attention_launches(q[0], kv, batch, **akw)
    launches_per_step = 1 + L * per_layer + launches_sampler + 1  # reserve, layers, sampler, commit
    if world > 1:
        t = torch.tensor([step_ms, e2e_ms, attn_ms, samp_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, e2e_ms, attn_ms, samp_ms = t.tolist()
        cnt = torch.tensor([committed, e2e_committed], device=device, dtype=torch.float64)
        dist.all_reduce(cnt)
        committed, e2e_committed = [int(x) for x in cnt.tolist()]
    del graph, attn_graph
    kern = attention_kernel(q[0], kv, batch, **akw)
    return dict(kernel=kern, step_ms=step_ms, e2e_ms=e2e_ms, attn_ms=attn_ms, attn_bytes=attn_bytes, samp_ms=samp_ms,
                samp_bytes=samp_bytes, clocks=clk, h2d=h2d, d2h=d2h, launches=launches_per_step * args.steps,
                committed=committed, e2e_committed=e2e_committed, e2e_steps=e2e_steps,
                tokens_per_round=committed / float(args.steps * B * world))


UMMA_FLAG = {"auto": 0, "mma": -1, "tcgen05": 1}
LAYOUT_FLAG = {"auto": 0, "keys": 1, "rows": 2, "direct": 3}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: c4 20 slices of the request stream, c2/c3/c5 400)")
    ap.add_argument("--warmup", type=int, default=None, help="untimed warm-up steps (default: c4 3, others 10)")
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--attn-kernel", choices=["auto", "mma", "tcgen05"], default="auto",
                    help="paged attention kernel: the library's automatic choice (default), the mma.sync "
                         "split-K kernel or the persistent tcgen05 kernel")
    ap.add_argument("--mma-layout", choices=["auto", "keys", "rows", "direct"], default="auto",
                    help="mma.sync kernel layout: the library's automatic choice (default), keys or query rows "
                         "on the MMA M dimension")
    ap.add_argument("--append", choices=["fused", "separate"], default="fused",
                    help="store each layer's new K/V rows inside the attention launch (default) or with a "
                         "separate append launch before it")
    ap.add_argument("--workload", choices=["c2", "c3", "c4", "c5", "c4attn"], default="c4",
                    help="c4: continuous-batching spec scheduler end to end (default, the spec-decode "
                         "tokens/s headline); c2: decode attention + KV append; c3: verify step at gamma=5; "
                         "c5: the attention of one long-context round at gamma=6 (draft decodes + target verify); "
                         "c4attn: C4's two attention ops alone at --batch sequences of C4 contexts (a profiling "
                         "target, one JSON line per op)")
    ap.add_argument("--requests", type=int, default=2048,
                    help="c4: requests in the whole job's arrival stream (the config's 2048)")
    ap.add_argument("--eager", action="store_true", help="c4: run the model forwards eagerly instead of CUDA graphs")
    ap.add_argument("--kernel-table", type=str, default=None, metavar="A:B",
                    help="c4: record rounds A..B of the warm-up run with torch.profiler (CUPTI) and print each "
                         "kernel's time per round and share of the GPU time to stderr")
    ap.add_argument("--overlap-layers", choices=["auto", "on", "off"], default="auto",
                    help="c2/c3/c5: consecutive layers' attention launches overlap (sdl_attn_args.overlap_layers); "
                         "auto: on for c2 and c5 (measured faster), off for c3 (measured slower)")
    ap.add_argument("--exact-plan", action="store_true",
                    help="c4attn: plan with the exact key count instead of the captured forwards' ragged plan")
    ap.add_argument("--no-batch-prefill", action="store_true",
                    help="c4: prefill same-round arrivals one by one (graph replays) instead of one chunked batch")
    ap.add_argument("--layers", type=int, default=None,
                    help="fewer layers only for profiling captures (default: the workload's model depth)")
    ap.add_argument("--batch", type=int, default=None, help="sequences per GPU (C2: 64, C3: 32)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    if args.steps is None:
        args.steps = 20 if args.workload in ("c4", "c4attn") else 400
    if args.warmup is None:
        args.warmup = 3 if args.workload in ("c4", "c4attn") else 10
    if args.warmup < 3:
        args.warmup = 3
    if args.batch is None:
        args.batch = {"c2": C2["batch"], "c3": C3["batch"], "c5": C5["batch"]}.get(args.workload, args.requests)
    if args.workload == "c5":
        return main_c5(args)
    if args.workload == "c4":
        return main_c4(args)
    if args.workload == "c4attn":
        return main_c4attn(args)
    if args.layers is None:
        args.layers = 28
    if args.workload == "c3":
        return main_c3(args)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = {"workload": "C2: paged decode attention + KV append (Qwen2.5-1.5B attention shapes)",
           "layers": args.layers, "q_heads": C2["q_heads"], "kv_heads": C2["kv_heads"], "head_dim": C2["head_dim"],
           "block_size": C2["block_size"], "batch_per_gpu": args.batch, "global_batch": args.batch * world,
           "ctx": "U[{},{}] seeded per rank".format(C2["ctx_lo"], C2["ctx_hi"]),
           "block_tables": "random permutation of a pool holding every context",
           "l2": "no flush needed: each attention launch reads ~151 MB of K/V (> 126 MB L2), layers disjoint",
           "parallelism": "dp{} (request-sharded, independent KV pools)".format(world),
           "attention_kernel": args.attn_kernel, "mma_layout": args.mma_layout, "kv_append": args.append,
           "overlap_layers": _overlap_layers(args)}

    if args.impl == "reference":
        if rank != 0:
            return 0
        threads = os.cpu_count() or 1
        vals = []
        per = min(args.cpu_seconds, 150.0 / max(1, args.steps + args.warmup))
        base = CpuC2(seed=args.seed, threads=threads)
        for i in range(args.warmup + args.steps):
            r = base.measure(per)
            if i >= args.warmup:
                vals.append(r["value"])
        value = float(np.mean(vals))
        line = {"metric": METRIC, "value": round(value, 4), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 * per, 3),
                "step_meaning": "one bounded host sample of the workload ({:.2f} s; see cpu_baseline.sample); "
                                "a whole C2 step would take {:.0f} ms on the host".format(per, 1000.0 * args.batch / value),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64 (numpy port)",
                "data": "synthetic", "config": cfg, "impl": "reference",
                "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
                                 "sample": r["sample"]},
                "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the B200 path has no CPU fallback)")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    res = run_gpu(args, rank, world, device)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = CpuC2(seed=args.seed).measure(args.cpu_seconds)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    hbm, peak_kind = _peaks()
    achieved = res["attn_bytes"] / (res["attn_ms"] * 1e-3) / 1e9
    value = args.batch * world / (res["step_ms"] * 1e-3)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(res["step_ms"], 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) Q/K/V, U[512,4096] contexts, random-permutation block tables)",
        "config": cfg,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4),
                     "traffic": C2_ATTN_TRAFFIC if args.layers == 28 and res["kernel"] == "mma" else None,
                     "traffic_source": "ncu --set full capture of attn_tc_kernel on this workload (dram read + "
                                       "write per launch, main kernel only; summary under profiles/)",
                     "kernel": ATTN_KERNELS[res["kernel"]] +
                               " (one paged decode attention op per layer{})".format(
                                   ", new K/V row stored inside it" if args.append == "fused" else ""),
                     "algorithmic_bytes_per_launch": res["attn_bytes"], "ms_per_launch": round(res["attn_ms"], 5),
                     "peak_source": "{} (MEASURED_PEAKS.json hbm_gbs)".format(peak_kind)},
        "e2e": {"value": round(args.batch * world / (res["e2e_ms"] * 1e-3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"],
                "path": ("public per-layer API (PagedKVCache.reserve/release + paged_attention{}), pinned host "
                         "I/O on a copy stream pipelined with the layers (step s+1's inputs up and step s-1's "
                         "outputs down while step s computes)").format(
                    " with k_new/v_new" if args.append == "fused" else " after PagedKVCache.append")},
        "gpu_launches": res["launches"],
        "clocks": res["clocks"],
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


def main_c3(args) -> int:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    c = C3
    cfg = {"workload": "C3: verify step at gamma=5 (extend attention + fused rejection sampling + rewind)",
           "layers": args.layers, "q_heads": c["q_heads"], "kv_heads": c["kv_heads"], "head_dim": c["head_dim"],
           "block_size": c["block_size"], "gamma": c["gamma"], "vocab": c["vocab"], "temperature": c["temperature"],
           "batch_per_gpu": args.batch, "global_batch": args.batch * world,
           "ctx": "U[{},{}] seeded per rank".format(c["ctx_lo"], c["ctx_hi"]),
           "logits": "N(0, 2) fp32, target gamma+1 rows and draft gamma rows per sequence",
           "block_tables": "random permutation of a pool holding every context",
           "l2": "no flush needed: a step streams ~1.06 GB of K/V over 28 disjoint layers and 214 MB of logits",
           "parallelism": "dp{} (request-sharded, independent KV pools)".format(world),
           "attention_kernel": args.attn_kernel, "mma_layout": args.mma_layout, "kv_append": args.append,
           "overlap_layers": _overlap_layers(args)}
    if args.impl == "reference":
        if rank != 0:
            return 0
        threads = os.cpu_count() or 1
        per = min(args.cpu_seconds, 150.0 / max(1, args.steps + args.warmup))
        base = CpuC3(seed=args.seed, threads=threads, batch=args.batch)
        vals = []
        for i in range(args.warmup + args.steps):
            r = base.measure(per)
            if i >= args.warmup:
                vals.append(r["value"])
        value = float(np.mean(vals))
        line = {"metric": METRIC, "value": round(value, 4), "unit": "tokens/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 * per, 3),
                "step_meaning": "one bounded host sample of the workload ({:.2f} s; see cpu_baseline.sample)".format(per),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (attention f64)",
                "data": "synthetic", "config": cfg, "impl": "reference",
                "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
                                 "sample": r["sample"]},
                "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the B200 path has no CPU fallback)")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    res = run_gpu_c3(args, rank, world, device)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = CpuC3(seed=args.seed, batch=args.batch).measure(args.cpu_seconds)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    hbm, peak_kind = _peaks()
    achieved = res["attn_bytes"] / (res["attn_ms"] * 1e-3) / 1e9
    samp_gbs = res["samp_bytes"] / (res["samp_ms"] * 1e-3) / 1e9
    value = res["committed"] / (args.steps * res["step_ms"] * 1e-3)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(res["step_ms"], 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) Q/K/V, N(0,2) logits, U[256,2048] contexts, random-permutation tables)",
        "config": cfg,
        "tokens_per_round": round(res["tokens_per_round"], 4),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(achieved / hbm, 4), "traffic": None,
                     "kernel": ATTN_KERNELS[res["kernel"]] +
                               ": (gamma+1)-row verify attention{}".format(
                                   ", new K/V rows stored inside it" if args.append == "fused" else ""),
                     "algorithmic_bytes_per_launch": res["attn_bytes"], "ms_per_launch": round(res["attn_ms"], 5),
                     "peak_source": "{} (MEASURED_PEAKS.json hbm_gbs)".format(peak_kind)},
        "sampler": {"achieved": round(samp_gbs, 1), "unit": "GB/s", "frac": round(samp_gbs / hbm, 4),
                    "algorithmic_bytes": res["samp_bytes"], "ms": round(res["samp_ms"], 5),
                    "kernels": "stats_kernel + accept_logits_kernel + wsum_kernel + finish_kernel "
                               "(sdl_spec_sample_logits)"},
        "e2e": {"value": round(res["e2e_committed"] / (res["e2e_steps"] * res["e2e_ms"] * 1e-3), 2),
                "unit": "tokens/s", "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"],
                "path": "public API (PagedKVCache.reserve, paged_attention {}, spec_sample_logits, "
                        "sdl_spec_commit), pinned host Q/K/V, logits and proposals in on a copy stream pipelined "
                        "with the previous step's compute, tokens and accept lengths out".format(
                            "with k_new/v_new" if args.append == "fused" else "after PagedKVCache.append")},
        "gpu_launches": res["launches"],
        "clocks": res["clocks"],
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


def run_gpu_c5(args, rank: int, world: int, device):
    """The attention of one C5 round on one GPU: gamma draft decode steps over
    the draft's layers, then the (gamma+1)-row verify over the target's
    layers, each layer one fused append + attention launch; both caches are
    rewound to the context afterwards."""
    import torch

    from engine import _lib
    from engine.attention import AttnBatch, attention_kernel, attention_launches, paged_attention
    from engine.kv import PagedKVCache
    from engine.workloads import c2_layout

    c = C5
    akw = dict(use_umma=UMMA_FLAG[args.attn_kernel], mma_layout=LAYOUT_FLAG[args.mma_layout],
               overlap_layers=_overlap_layers(args))
    Lt = args.layers or c["target_layers"]
    Ld = args.layers or c["draft_layers"]
    B, gam, Hkv, d, bs = args.batch, c["gamma"], c["kv_heads"], c["head_dim"], c["block_size"]
    Hqt, Hqd = c["target_q_heads"], c["draft_q_heads"]
    seed = args.seed + rank
    ctx, _, _ = c2_layout(seed, B, c["ctx_lo"], c["ctx_hi"], bs)
    sids = list(range(B))
    gd = torch.Generator(device=device)
    gd.manual_seed(seed)

    def make_cache(L, extra):
        cap = sum(-(-(x + extra) // bs) for x in ctx) + B
        kv = PagedKVCache(L, Hkv, d, cap, bs, device, torch.bfloat16,
                          max_blocks_per_seq=-(-(c["ctx_hi"] + extra + 1) // bs), max_seqs=B)
        g = torch.Generator(device="cpu")
        g.manual_seed(seed + L)
        kv.allocator._free_stack.copy_(torch.randperm(cap, generator=g).to(torch.int32))
        for sid in sids:
            kv.add_sequence(sid)
        kv.reserve(sids, [0] * B, ctx)
        kv._k.normal_(generator=gd)
        kv._v.normal_(generator=gd)
        return kv

    tgt = make_cache(Lt, gam + 1)
    dft = make_cache(Ld, gam)
    bf = torch.bfloat16
    qt = torch.randn((Lt, B, gam + 1, Hqt, d), generator=gd, device=device).to(bf)
    kt = torch.randn((Lt, B * (gam + 1), Hkv, d), generator=gd, device=device).to(bf)
    vt = torch.randn((Lt, B * (gam + 1), Hkv, d), generator=gd, device=device).to(bf)
    qd = torch.randn((gam, Ld, B, 1, Hqd, d), generator=gd, device=device).to(bf)
    kd = torch.randn((gam, Ld, B, Hkv, d), generator=gd, device=device).to(bf)
    vd = torch.randn((gam, Ld, B, Hkv, d), generator=gd, device=device).to(bf)
    ot = torch.empty_like(qt)
    od = torch.empty_like(qd)
    vbatch = AttnBatch.from_lists(device, sids, ctx, gam + 1)
    dbatches = [AttnBatch.from_lists(device, sids, [x + s for x in ctx], 1) for s in range(gam)]
    rel = [_lib.REL_TRUNCATE] * B

    def draft_layers():
        for s in range(gam):
            for layer in range(Ld):
                paged_attention(qd[s, layer], dft, layer, dbatches[s], out=od[s, layer], **akw,
                                k_new=kd[s, layer], v_new=vd[s, layer])

    def verify_layers():
        for layer in range(Lt):
            paged_attention(qt[layer], tgt, layer, vbatch, out=ot[layer], **akw, k_new=kt[layer],
                            v_new=vt[layer])

    def reserve():
        tgt.reserve(sids, ctx, [gam + 1] * B)
        dft.reserve(sids, ctx, [gam] * B)

    def release():
        tgt.release(sids, ctx, rel)
        dft.release(sids, ctx, rel)

    reserve()
    draft_layers()
    verify_layers()
    release()
    torch.cuda.synchronize(device)
    g_draft, g_verify = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
    with torch.cuda.graph(g_draft):
        draft_layers()
    with torch.cuda.graph(g_verify):
        verify_layers()
    torch.cuda.synchronize(device)
    stream = torch.cuda.current_stream(device)

    def device_step():
        reserve()
        g_draft.replay()
        g_verify.replay()
        release()

    for _ in range(args.warmup):
        device_step()
    torch.cuda.synchronize(device)
    tgt.check_errors()
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    clocks = ClockSampler(device.index if device.index is not None else 0) if rank == 0 else None
    if clocks:
        clocks.start()
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        device_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    step_ms = e0.elapsed_time(e1) / args.steps

    # per-kernel rooflines: the draft decode graph and the verify graph alone
    reps = max(3, args.steps // 4)
    reserve()
    timings = {}
    for name, gr, n in (("draft", g_draft, gam * Ld), ("verify", g_verify, Lt)):
        gr.replay()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(reps):
            gr.replay()
        a1.record(stream)
        torch.cuda.synchronize(device)
        timings[name] = a0.elapsed_time(a1) / (reps * n)
    release()
    clk = clocks.stop() if clocks else None
    tgt.check_errors()
    dft.check_errors()

    # e2e: the same round through the public per-layer API without graphs,
    # new Q/K/V rows from pinned host memory, outputs back every round
    hq = [t.cpu().pin_memory() for t in (qt, kt, vt, qd, kd, vd)]
    oth = torch.empty(ot.shape, dtype=bf).pin_memory()
    odh = torch.empty(od.shape, dtype=bf).pin_memory()
    h2d = sum(t.numel() * 2 for t in hq)
    d2h = (oth.numel() + odh.numel()) * 2

    def e2e_step():
        q_t, k_t, v_t, q_d, k_d, v_d = (t.to(device, non_blocking=True) for t in hq)
        reserve()
        for s in range(gam):
            for layer in range(Ld):
                paged_attention(q_d[s, layer], dft, layer, dbatches[s], out=od[s, layer], **akw,
                                k_new=k_d[s, layer], v_new=v_d[s, layer])
        for layer in range(Lt):
            paged_attention(q_t[layer], tgt, layer, vbatch, out=ot[layer], **akw, k_new=k_t[layer],
                            v_new=v_t[layer])
        odh.copy_(od, non_blocking=True)
        oth.copy_(ot, non_blocking=True)
        release()

    e2e_steps = max(3, args.steps // 4)
    e2e_step()
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    torch.cuda.synchronize(device)
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / e2e_steps

    vbytes = sum((x + gam + 1) * 2 * Hkv * d * 2 for x in ctx) + 2 * B * (gam + 1) * Hqt * d * 2 + \
        sum(-(-(x + gam + 1) // bs) * 4 for x in ctx) + 2 * B * (gam + 1) * 2 * Hkv * d * 2
    # one draft launch, averaged over the gamma steps (step s attends ctx + s + 1 keys)
    dbytes = (sum((x + 1 + s) * 2 * Hkv * d * 2 + -(-(x + 1 + s) // bs) * 4 for x in ctx for s in range(gam)) / gam
              + 2 * B * Hqd * d * 2 + 2 * B * 2 * Hkv * d * 2)
    launches = 2 + 2 + gam * Ld * attention_launches(qd[0, 0], dft, dbatches[0], **akw, k_new=kd[0, 0],
                                                     v_new=vd[0, 0]) + \
        Lt * attention_launches(qt[0], tgt, vbatch, **akw, k_new=kt[0], v_new=vt[0])
    kern = {"verify": attention_kernel(qt[0], tgt, vbatch, **akw),
            "draft": attention_kernel(qd[0, 0], dft, dbatches[0], **akw)}
    if world > 1:
        t = torch.tensor([step_ms, e2e_ms, timings["draft"], timings["verify"]], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, e2e_ms, timings["draft"], timings["verify"] = t.tolist()
    del g_draft, g_verify
    return dict(kernel=kern, step_ms=step_ms, e2e_ms=e2e_ms, verify_ms=timings["verify"], draft_ms=timings["draft"],
                verify_bytes=vbytes, draft_bytes=dbytes, clocks=clk, h2d=h2d, d2h=d2h,
                launches=launches * args.steps)


def main_c5(args) -> int:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    c = C5
    cfg = {"workload": "C5: attention of one long-context speculative round at gamma=6 "
                       "(6 draft decode steps x 28 layers of the 1.5B shape, then the 7-row verify x 36 layers "
                       "of the 3B shape; K/V append fused into every launch)",
           "target_layers": args.layers or c["target_layers"], "draft_layers": args.layers or c["draft_layers"],
           "target_q_heads": c["target_q_heads"], "draft_q_heads": c["draft_q_heads"], "kv_heads": c["kv_heads"],
           "head_dim": c["head_dim"], "block_size": c["block_size"], "gamma": c["gamma"],
           "batch_per_gpu": args.batch, "global_batch": args.batch * world,
           "ctx": "U[{},{}] seeded per rank".format(c["ctx_lo"], c["ctx_hi"]),
           "tokens": "verified positions per round, batch x (gamma+1): the round's upper bound on committed "
                     "tokens (models and acceptance not modelled)",
           "block_tables": "random permutation of a pool holding every context",
           "l2": "no flush needed: every launch reads ~337 MB of K/V (> 126 MB L2)",
           "parallelism": "dp{} (request-sharded, independent KV pools)".format(world),
           "attention_kernel": args.attn_kernel, "mma_layout": args.mma_layout,
           "overlap_layers": _overlap_layers(args)}
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "metric": METRIC, "config": cfg,
                              "unavailable": "C5 is not timed on the CPU port (one C5 layer of the numpy port "
                                             "takes minutes); the C2 and C3 lines carry the CPU baseline"}))
        return 0

    import torch

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the B200 path has no CPU fallback)")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    res = run_gpu_c5(args, rank, world, device)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    hbm, peak_kind = _peaks()
    tokens = args.batch * world * (c["gamma"] + 1)
    v_gbs = res["verify_bytes"] / (res["verify_ms"] * 1e-3) / 1e9
    d_gbs = res["draft_bytes"] / (res["draft_ms"] * 1e-3) / 1e9
    names = ATTN_KERNELS
    line = {
        "metric": METRIC,
        "value": round(tokens / (res["step_ms"] * 1e-3), 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(res["step_ms"], 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) Q/K/V, U[8192,32768] contexts, random-permutation block tables)",
        "config": cfg,
        "roofline": {"bound": "hbm", "achieved": round(v_gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(v_gbs / hbm, 4), "traffic": None,
                     "kernel": names[res["kernel"]["verify"]] + ": 7-row verify attention (3B shape)",
                     "algorithmic_bytes_per_launch": res["verify_bytes"], "ms_per_launch": round(res["verify_ms"], 5),
                     "peak_source": "{} (MEASURED_PEAKS.json hbm_gbs)".format(peak_kind)},
        "decode_roofline": {"achieved": round(d_gbs, 1), "peak": hbm, "unit": "GB/s", "frac": round(d_gbs / hbm, 4),
                            "kernel": names[res["kernel"]["draft"]] + ": draft decode attention (1.5B shape)",
                            "algorithmic_bytes_per_launch": res["draft_bytes"],
                            "ms_per_launch": round(res["draft_ms"], 5)},
        "e2e": {"value": round(tokens / (res["e2e_ms"] * 1e-3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"],
                "path": "public per-layer API (PagedKVCache.reserve/release + paged_attention with k_new/v_new), "
                        "no graphs, pinned host Q/K/V in and attention outputs out"},
        "cpu_baseline": None,
        "gpu_launches": res["launches"],
        "clocks": res["clocks"],
    }
    print(json.dumps(line), flush=True)
    return 0


def _time_attention_op(device, ctx, chunk, Hq, Hkv, d, layers, seed, reps, span_cap=None, **akw):
    """One attention op as a model forward launches it -- the K/V rows of
    ``chunk`` new positions stored inside the paged attention launch -- over
    contexts ``ctx`` (a random-permutation pool of exactly those pages), timed
    with CUDA events over ``reps`` replays of a graph of ``layers`` launches.
    With ``span_cap`` (the block-table width in tokens of the serving pools)
    the call carries what a captured model forward passes: the key-span
    bucket as max_limit and no key count (ragged rows, key_count < 0), so the
    plan is the one the C4 run's graphs replay; without it, the exact key
    count.  Returns the kernel name, ms per launch and algorithmic bytes per
    launch."""
    import torch

    from engine.attention import AttnBatch, attention_kernel, attention_launches, paged_attention
    from engine.kv import PagedKVCache

    bs = 16
    B = len(ctx)
    cap = sum(-(-(x + chunk) // bs) for x in ctx) + B
    width = max(-(-(x + chunk) // bs) for x in ctx) + 1
    span = None
    if span_cap is not None:
        span = 1024
        while span < max(ctx) + chunk:
            span *= 2
        span = min(span, int(span_cap))
        width = max(width, -(-span // bs))
    kv = PagedKVCache(layers, Hkv, d, cap, bs, device, torch.bfloat16, max_blocks_per_seq=width, max_seqs=B)
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    kv.allocator._free_stack.copy_(torch.randperm(cap, generator=g).to(torch.int32))
    sids = list(range(B))
    for sid in sids:
        kv.add_sequence(sid)
    kv.reserve(sids, [0] * B, ctx)
    gd = torch.Generator(device=device)
    gd.manual_seed(seed)
    kv._k.normal_(generator=gd)
    kv._v.normal_(generator=gd)
    bf = torch.bfloat16
    q = torch.randn((layers, B, chunk, Hq, d), generator=gd, device=device).to(bf)
    kn = torch.randn((layers, B * chunk, Hkv, d), generator=gd, device=device).to(bf)
    vn = torch.randn((layers, B * chunk, Hkv, d), generator=gd, device=device).to(bf)
    out = torch.empty_like(q)
    batch = AttnBatch.from_lists(device, sids, ctx, chunk)
    if span is not None:
        batch = AttnBatch(batch.rows, batch.starts, span, key_count=-1)
    kv.reserve(sids, ctx, [chunk] * B)

    def run():
        for layer in range(layers):
            paged_attention(q[layer], kv, layer, batch, out=out[layer], k_new=kn[layer], v_new=vn[layer], **akw)

    run()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        run()
    stream = torch.cuda.current_stream(device)
    graph.replay()
    graph.replay()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(reps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(device)
    kv.check_errors()
    ms = e0.elapsed_time(e1) / (reps * layers)
    nbytes = (sum((x + chunk) * 2 * Hkv * d * 2 for x in ctx) + 2 * B * chunk * Hq * d * 2
              + sum(-(-(x + chunk) // bs) * 4 for x in ctx) + 2 * (B * chunk * 2 * Hkv * d * 2))
    kern = attention_kernel(q[0], kv, batch, **akw)
    launches = attention_launches(q[0], kv, batch, k_new=kn[0], v_new=vn[0], **akw)
    del graph
    return {"kernel": kern, "ms": ms, "bytes": nbytes, "launches_per_op": launches, "batch": B,
            "mean_ctx": round(sum(ctx) / max(1, B), 1), "plan": "exact key count" if span is None else
            "ragged rows, span {} (the captured forwards' plan)".format(span)}


def _print_kernel_table(p, rounds, wall_s, b0, b1) -> None:
    """Kernel time per round and share of the GPU time (CUPTI activity of a
    torch.profiler window), with the GPU-busy fraction of the window."""
    import collections

    import torch

    evs = [e for e in p.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    spans = sorted((e.time_range.start, e.time_range.end) for e in evs)
    busy, cur = 0.0, None
    for a, b in spans:
        if cur is None or a > cur[1]:
            if cur:
                busy += cur[1] - cur[0]
            cur = [a, b]
        else:
            cur[1] = max(cur[1], b)
    if cur:
        busy += cur[1] - cur[0]
    agg = collections.defaultdict(lambda: [0, 0.0])
    for e in evs:
        k = e.name.replace("(anonymous namespace)::", "").split("(")[0][:80]
        agg[k][0] += 1
        agg[k][1] += e.time_range.end - e.time_range.start
    tot = sum(v[1] for v in agg.values()) or 1.0
    out = sys.stderr
    print("kernel table: {} rounds (batch {} -> {}), wall {:.2f} ms/round, GPU busy {:.2f} ms/round ({:.0%})".format(
        rounds, b0, b1, 1e3 * wall_s / rounds, busy / 1e3 / rounds, busy / 1e3 / (1e3 * wall_s)), file=out)
    for k, (n, t) in sorted(agg.items(), key=lambda kv: -kv[1][1])[:30]:
        print("  {:8.3f} ms/round {:5.1f}%  {:6d} launches  {}".format(t / 1e3 / rounds, 100 * t / tot, n, k), file=out)


def _overlap_layers(args) -> bool:
    """Whether the attention-stack workloads launch their layers with
    sdl_attn_args.overlap_layers: each launch lets the next layer's become
    resident at its start and streams its older pages before the dependency
    wait.  The contract holds here: consecutive launches are distinct layers,
    and a layer's own appends of the previous step are complete (or store
    the same bytes again) before it is read.  Measured on B200: C2 decode
    30.5 -> 28.9 us per layer, C5 round 13.91 -> 13.62 ms; C3 verify 19.3 ->
    20.2 us (its three 6-warp CTAs per SM leave no slot for the next layer
    until the tail), so auto keeps it off there."""
    if args.overlap_layers != "auto":
        return args.overlap_layers == "on"
    return args.workload in ("c2", "c5")


def main_c4attn(args) -> int:
    """C4's attention ops alone (one GPU): the 0.5B-shaped draft decode
    (14 q / 2 kv heads, head_dim 64) and the 1.5B-shaped 5-row verify (12 q
    heads, head_dim 128), each with its K/V append fused, over ``--batch``
    sequences whose contexts follow C4's prompt distribution plus up to 300
    generated tokens; ``--layers`` layers per graph (default 8), ``--steps``
    graph replays.  Prints one JSON line per op (not a bench line: a
    profiling target for the batch sizes a C4 run reaches)."""
    import torch

    from engine import workloads

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the B200 path has no CPU fallback)")
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    c = workloads.C4
    rng = np.random.default_rng(args.seed)
    ctx = [int(min(c["prompt_cap"], max(16, np.floor(rng.lognormal(c["prompt_mu"], c["prompt_sigma"])))))
           + int(rng.integers(0, 300)) for _ in range(args.batch)]
    akw = dict(use_umma=UMMA_FLAG[args.attn_kernel], mma_layout=LAYOUT_FLAG[args.mma_layout])
    hbm, _ = _peaks()
    layers = args.layers or 8
    # the C4 pools' block-table width in tokens (prompt cap + output cap), as the run's graphs see it
    span_cap = None if args.exact_plan else ((c["prompt_cap"] + c["out_hi"] + 16) // 16 + 2) * 16
    for name, chunk, Hq, d in (("draft decode (0.5B shape)", 1, 14, 64), ("5-row verify (1.5B shape)", 5, 12, 128)):
        r = _time_attention_op(device, ctx, chunk, Hq, 2, d, layers, args.seed + 7, max(1, args.steps),
                               span_cap=span_cap, **akw)
        gbs = r["bytes"] / (r["ms"] * 1e-3) / 1e9
        print(json.dumps({"op": name, "batch": args.batch, "mean_ctx": r["mean_ctx"], "plan": r["plan"],
                          "kernel": ATTN_KERNELS[r["kernel"]],
                          "us_per_launch": round(r["ms"] * 1e3, 2), "algorithmic_mb": round(r["bytes"] / 1e6, 1),
                          "gbs": round(gbs, 1), "frac_of_measured_hbm": round(gbs / hbm, 4)}), flush=True)
    return 0


def main_c4(args) -> int:
    """C4: the continuous-batching speculative
    scheduler end to end on random-init Qwen2.5-1.5B (target) / 0.5B (draft)
    shaped bf16 models, gamma=4, temperature 1.0, KV pools sized to 80 % of
    the free HBM.  The metric is the reference's own: generated tokens /
    makespan (engine/scheduler.py:81-84), summed over ranks / slowest rank.

    One global stream of ``--requests`` (2048) requests with Poisson arrivals
    at 64 requests/s per GPU is sharded round-robin over the ranks
    (``engine.distributed.shard_requests``) and served by one continuous run
    per rank: a request is admitted at the first round boundary after its
    wall-clock arrival, and the run ends when the last request finishes.  A
    *step* is one of ``--steps`` equal slices of that stream (the timed
    region serves all of them back to back, without draining in between, as
    a server would), so ms_per_step = makespan / steps.  Before timing: every
    CUDA graph is captured up front (``capture_graphs``, independent of the
    requests) and ``--warmup`` slices' worth of a different request stream
    is served."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    from engine import workloads

    c = workloads.C4
    total = args.requests
    K, W = args.steps, args.warmup
    rate = c["arrival_rate"] * world
    cfg = {"workload": "C4: continuous-batching speculative scheduler, gamma=4, T=1.0 (Qwen2.5-1.5B target / "
                       "0.5B draft shapes, random-init bf16 weights)",
           "global_requests": total,
           "requests_per_step": "{}/{} (a step is a slice of the one arrival stream; the stream is served by one "
                                "continuous run per rank, sharded round-robin)".format(total, K),
           "prompts": "floor(lognormal(6, 0.8)) capped at 4096, ids U[0, 151936)",
           "outputs": "U[64, 512] new tokens",
           "arrivals": "Poisson, 64 requests/s per GPU ({:g}/s for the whole job), wall clock: a request is "
                       "admitted at the first round boundary after its arrival".format(rate),
           "kv_pool": "80% of free HBM after weights, block_size 16, target and draft pools; recompute "
                      "preemption when a round would not fit (per_rank.preempted counts it)",
           "forwards": "eager" if args.eager else "CUDA-graph replays, all captured before the warm-up: a round's "
                                                  "gamma draft steps as one graph, the verify forward, and the "
                                                  "prefill chunk-row buckets (batch x key-span buckets; attention "
                                                  "plans for ragged rows)",
           "admission": ("one prefill per arrival" if args.no_batch_prefill else
                         "same-round arrivals prefilled together in 128-token chunks (one forward per model)"),
           "warmup": "{} requests of a different stream (seed {})".format(max(1, (total * W) // K), args.seed + 1000003),
           "l2": "no flush needed: weights (4.1 GB) and the KV pages of a round are far larger than L2",
           "parallelism": "dp{} (request-sharded, independent engines and KV pools)".format(world)}
    if args.impl == "reference":
        if rank != 0:
            return 0
        threads = os.cpu_count() or 1
        per = max(2.0, min(args.cpu_seconds, 150.0 / max(1, K + W)))
        base = CpuC4(seed=args.seed, threads=threads)
        vals, samples = [], []
        for i in range(W + K):
            r = base.measure(per)
            if i >= W:
                vals.append(r["value"])
                samples.append(r["sample_seconds"])
        value = float(np.mean(vals))
        line = {"metric": METRIC, "value": round(value, 4), "unit": "tokens/s", "n_gpus": world,
                "steps": K, "warmup": W, "ms_per_step": round(1000.0 * float(np.mean(samples)), 3),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "f32 (attention f64)", "data": "synthetic", "config": cfg, "impl": "reference",
                "step_meaning": "one bounded host sample of the C4 scheduler (see cpu_baseline.sample); "
                                "ms_per_step is the host time a sample took",
                "cpu_baseline": {"value": round(value, 4), "unit": "tokens/s", "cores": threads, "kind": "port",
                                 "sample": r["sample"]},
                "e2e": {"value": round(value, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return 0

    import torch

    from engine import _lib
    from engine.config import EngineConfig, WorkloadRequest
    from engine.distributed import gather_results, init_from_env, shard_requests
    from engine.qwen import build_random_model
    from engine.scheduler import build_kv
    from engine.spec_scheduler import SpeculativePagedScheduler
    from specdec.config import SamplingConfig as SpecSampling

    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device (the B200 path has no CPU fallback)")
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    init_from_env("nccl" if world > 1 else None, timeout_s=600.0)
    dist = None
    if world > 1:
        import torch.distributed as dist
    bf = torch.bfloat16
    tcfg = workloads.shape_config(c["target"], max_position_embeddings=8192)
    dcfg = workloads.shape_config(c["draft"], max_position_embeddings=8192)
    target = build_random_model(tcfg, device, bf, seed=1)
    draft = build_random_model(dcfg, device, bf, seed=2)

    def stream_of(seed, n):
        """This rank's share of an ``n``-request arrival stream (global arrival times)."""
        return shard_requests(workloads.c4_requests_wall(seed, n, rate, c["vocab"]), rank, world, "round_robin")

    timed = stream_of(args.seed, total)
    warm = stream_of(args.seed + 1000003, max(1, (total * W) // K))
    per_run = max(len(timed), len(warm))
    free, _ = torch.cuda.mem_get_info(device)
    per_block = 16 * 2 * 2 * (target.num_layers * target.num_kv_heads * target.head_dim +
                              draft.num_layers * draft.num_kv_heads * draft.head_dim)
    blocks = int(c["pool_fraction"] * free / per_block)
    ecfg = EngineConfig(block_size=16, max_num_blocks=blocks, max_batch=per_run)
    width = (c["prompt_cap"] + c["out_hi"] + 16) // 16 + 2
    kv = build_kv(target, ecfg, device, max_blocks_per_seq=width, max_seqs=per_run + 2)
    dkv = build_kv(draft, ecfg, device, max_blocks_per_seq=width, max_seqs=per_run + 2)
    if not args.eager:
        target.enable_cuda_graphs()
        draft.enable_cuda_graphs()
    sched = SpeculativePagedScheduler(target, kv, draft, dkv, ecfg, SpecSampling(temperature=c["temperature"]),
                                      c["gamma"])
    sched.preemption = "recompute"  # a full pool parks and later re-prefills sequences instead of raising
    sched.batch_prefill = not args.no_batch_prefill
    t_cap = time.perf_counter()
    n_graphs = sched.capture_graphs()
    cap_s = time.perf_counter() - t_cap
    first_sid = sched._next_sid  # rows from here on serve requests; every slice reuses them

    rounds = {"n": 0, "rows": 0, "max": None}

    def hook(sids, starts, d0):
        rounds["n"] += 1
        rounds["rows"] += len(sids)
        best = rounds["max"]
        if best is None or len(sids) * (1 + sum(starts) / len(sids)) > best[0]:
            rounds["max"] = (len(sids) * (1 + sum(starts) / len(sids)), list(starts), list(d0))

    def requests_of(part, staged):
        out = []
        for ids, new, t in part:
            prompt = torch.tensor(ids, dtype=torch.long).to(device) if staged else ids
            out.append(WorkloadRequest(prompt=prompt, max_new_tokens=new, arrive_time=t))
        return out

    def serve(reqs, seed):
        """One continuous run over ``reqs`` (wall-clock arrivals); returns generated tokens."""
        assert kv.num_allocated_blocks == 0 and dkv.num_allocated_blocks == 0
        sched._next_sid = first_sid
        return sched.run_spec_continuous(reqs, seed=seed, measure=False, arrival_clock="wall").generated_tokens

    prof = {}
    if args.kernel_table:
        lo, hi = (int(x) for x in args.kernel_table.split(":"))

        def prof_hook(sids, starts, d0):
            prof["n"] = prof.get("n", 0) + 1
            if prof["n"] == lo:
                torch.cuda.synchronize(device)
                prof["p"] = torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA])
                prof["p"].__enter__()
                prof["t0"] = time.perf_counter()
                prof["b0"] = len(sids)
            elif prof["n"] == hi:
                torch.cuda.synchronize(device)
                prof["wall"] = time.perf_counter() - prof["t0"]
                prof["p"].__exit__(None, None, None)
                prof["b1"] = len(sids)

        sched.round_hook = prof_hook
    serve(requests_of(warm, False), 7000)
    sched.round_hook = None
    torch.cuda.synchronize(device)
    kv.check_errors()
    dkv.check_errors()
    if "wall" in prof:
        _print_kernel_table(prof["p"], hi - lo, prof["wall"], prof["b0"], prof["b1"])

    # timed: prompts staged in HBM before the region (the "inputs resident" figure)
    staged = requests_of(timed, True)
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    clocks = ClockSampler(device.index if device.index is not None else 0) if rank == 0 else None
    if clocks:
        clocks.start()
    stream = torch.cuda.current_stream(device)
    calls0 = _lib.calls()
    sched.round_hook = hook
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    e0.record(stream)
    tokens = serve(staged, 100)
    e1.record(stream)
    torch.cuda.synchronize(device)
    ms = e0.elapsed_time(e1)
    preempted = sched.preemptions
    sched.round_hook = None
    calls = _lib.calls() - calls0
    clk = clocks.stop() if clocks else None
    kv.check_errors()
    dkv.check_errors()
    n_rounds, n_rows = rounds["n"], rounds["rows"]

    # e2e: the same public call with host prompt lists (copied up at admission)
    # over the same stream; token lists come back every round
    host = requests_of(timed, False)
    h2d = sum(len(r.prompt) * 8 for r in host)
    rounds_e = {"n": 0, "rows": 0}
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    sched.round_hook = lambda s, a, b: (rounds_e.__setitem__("n", rounds_e["n"] + 1),
                                        rounds_e.__setitem__("rows", rounds_e["rows"] + len(s)))
    e2e_tokens = serve(host, 100)
    torch.cuda.synchronize(device)
    e2e_ms = (time.perf_counter() - t0) * 1000.0
    sched.round_hook = None
    chunk = c["gamma"] + 1
    d2h = (rounds_e["rows"] * (chunk + 3) + 2 * rounds_e["n"]) * 4

    # kernel rooflines on the heaviest round's shapes (after freeing the pools)
    _, starts_max, d0_max = rounds["max"]
    del sched, kv, dkv
    torch.cuda.synchronize(device)
    torch.cuda.empty_cache()
    reps = 5
    span_cap = width * 16  # the pools' block-table width in tokens caps the graphs' key-span buckets
    draft_op = _time_attention_op(device, d0_max, 1, dcfg.num_attention_heads, dcfg.num_key_value_heads,
                                  dcfg.head_dim, dcfg.num_hidden_layers, args.seed + 5, reps, span_cap=span_cap)
    verify_op = _time_attention_op(device, starts_max, chunk, tcfg.num_attention_heads, tcfg.num_key_value_heads,
                                   tcfg.head_dim, tcfg.num_hidden_layers, args.seed + 6, reps, span_cap=span_cap)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = CpuC4(seed=args.seed).measure(args.cpu_seconds)
    payload = {"tokens": tokens, "ms": ms, "e2e_tokens": e2e_tokens, "e2e_ms": e2e_ms, "rounds": n_rounds,
               "rows": n_rows, "calls": calls, "draft_ms": draft_op["ms"], "verify_ms": verify_op["ms"],
               "preempted": preempted}
    allp = gather_results(payload)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    ms_max = max(p["ms"] for p in allp)
    tok_sum = sum(p["tokens"] for p in allp)
    e2e_max = max(p["e2e_ms"] for p in allp)
    e2e_sum = sum(p["e2e_tokens"] for p in allp)
    value = tok_sum / (ms_max * 1e-3)
    hbm, peak_kind = _peaks()
    d_ms = max(p["draft_ms"] for p in allp)
    v_ms = max(p["verify_ms"] for p in allp)
    d_gbs = draft_op["bytes"] / (d_ms * 1e-3) / 1e9
    v_gbs = verify_op["bytes"] / (v_ms * 1e-3) / 1e9
    names = ATTN_KERNELS
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms_max / K, 3),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded prompts, lengths and arrivals; random-init weights)",
        "config": cfg,
        "step_meaning": "one of {} equal slices of the arrival stream (served by one continuous run)".format(K),
        "generated_tokens": tok_sum,
        "makespan_ms": round(ms_max, 2),
        "per_rank": [{"tokens": p["tokens"], "ms": round(p["ms"], 1), "rounds": p["rounds"],
                      "mean_batch": round(p["rows"] / max(1, p["rounds"]), 2), "preempted": p["preempted"]}
                     for p in allp],
        "graphs_captured": n_graphs,
        "graph_capture_s": round(cap_s, 2),
        "roofline": {"bound": "hbm", "achieved": round(d_gbs, 1), "peak": hbm, "unit": "GB/s",
                     "frac": round(d_gbs / hbm, 4),
                     "traffic": round(draft_op["bytes"] * C4_DECODE_TRAFFIC_RATIO),
                     "traffic_source": "ncu dram read+write of attn_tc_kernel at 358 C4 sequences "
                                       "(profiles/attn_tc_kernel_c4_draft_decode_ragged.md), scaled by the "
                                       "algorithmic bytes of this launch",
                     "kernel": names[draft_op["kernel"]] + ": draft decode attention (0.5B shape, 24 layers), "
                               "K/V append fused, on the heaviest round's draft contexts",
                     "batch": draft_op["batch"], "mean_ctx": draft_op["mean_ctx"], "plan": draft_op["plan"],
                     "algorithmic_bytes_per_launch": draft_op["bytes"], "ms_per_launch": round(d_ms, 5),
                     "peak_source": "{} (MEASURED_PEAKS.json hbm_gbs)".format(peak_kind)},
        "verify_roofline": {"bound": "hbm", "achieved": round(v_gbs, 1), "peak": hbm, "unit": "GB/s",
                            "frac": round(v_gbs / hbm, 4),
                            "traffic": round(verify_op["bytes"] * C4_VERIFY_TRAFFIC_RATIO),
                            "traffic_source": "ncu dram read+write of attn_rows_kernel at 358 C4 sequences "
                                              "(profiles/attn_rows_kernel_c4_verify_ragged.md), scaled by the "
                                              "algorithmic bytes of this launch",
                            "kernel": names[verify_op["kernel"]] + ": 5-row verify attention (1.5B shape, 28 "
                                      "layers), K/V append fused, on the heaviest round's target contexts",
                            "batch": verify_op["batch"], "mean_ctx": verify_op["mean_ctx"],
                            "plan": verify_op["plan"],
                            "algorithmic_bytes_per_launch": verify_op["bytes"], "ms_per_launch": round(v_ms, 5)},
        "e2e": {"value": round(e2e_sum / (e2e_max * 1e-3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": round(h2d / K), "d2h_bytes_per_step": round(d2h / K),
                "path": "SpeculativePagedScheduler.run_spec_continuous over the same stream with host prompt "
                        "lists (copied up at admission) and host token lists out (one packed read per round), "
                        "host wall clock"},
        "gpu_launches": calls,
        "gpu_launches_note": "library entry calls in the timed region (graph replays counted with the calls "
                             "they captured); each launches one or two of this library's kernels",
        "clocks": clk,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
