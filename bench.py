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

Multi-GPU (torchrun): every rank runs its own batch of 64 sequences (weak
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


# --------------------------------------------------------------- GPU arm
def run_gpu(args, rank: int, world: int, device):
    import torch

    from engine import _lib
    from engine.attention import AttnBatch, attention_launches, paged_attention
    from engine.kv import PagedKVCache
    from engine.workloads import c2_layout

    c = dict(C2)
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
            if with_append:
                kv.append(layer, slots_static, knew[layer], vnew[layer])
            paged_attention(q[layer], kv, layer, batch, out=out[layer])

    # warm up every code path once outside capture (attributes, workspace)
    slots_static.copy_(kv.reserve(sids, ctx, [1] * B))
    step_layers()
    kv.release(sids, ctx, rel_flags)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):  # captured on torch's side stream, replayed on `stream`
        step_layers()
    attn_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(attn_graph):
        step_layers(with_append=False)
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

    def e2e_step():
        qd = q_h.to(device, non_blocking=True)
        kd = k_h.to(device, non_blocking=True)
        vd = v_h.to(device, non_blocking=True)
        slots = kv.reserve(sids, ctx, [1] * B)
        b2 = AttnBatch.from_lists(device, sids, ctx, 1)
        od = torch.empty_like(out)
        for layer in range(L):
            kv.append(layer, slots, kd[layer], vd[layer])
            paged_attention(qd[layer], kv, layer, b2, out=od[layer])
        o_h.copy_(od, non_blocking=True)
        kv.release(sids, ctx, rel_flags)

    e2e_steps = max(3, args.steps // 4)
    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize(device)
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        e2e_step()
    torch.cuda.synchronize(device)
    e2e_ms = (time.perf_counter() - t0) * 1000.0 / e2e_steps
    kv.check_errors()
    # parity spot-check: the public-API outputs equal the graph path's, bit for bit
    device_step()
    torch.cuda.synchronize(device)
    if not torch.equal(o_h.to(device), out):
        raise RuntimeError("e2e outputs differ from the graph path")

    attn_bytes = sum((x + 1) * 2 * Hkv * d * 2 for x in ctx) + 2 * B * Hq * d * 2 + sum(-(-(x + 1) // bs) * 4 for x in ctx)
    per_layer = 1 + attention_launches(q[0], kv, batch)  # append + attention (+ split merge)
    launches_per_step = 2 + L * per_layer  # + reserve + release
    if world > 1:
        t = torch.tensor([step_ms, e2e_ms, attn_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        step_ms, e2e_ms, attn_ms = t.tolist()
    del graph, attn_graph
    return dict(step_ms=step_ms, e2e_ms=e2e_ms, attn_ms=attn_ms, attn_bytes=attn_bytes, clocks=clk, h2d=h2d,
                d2h=d2h, launches=launches_per_step * args.steps, ctx_mean=float(np.mean(ctx)))


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--layers", type=int, default=C2["layers"], help="fewer layers only for profiling captures")
    ap.add_argument("--batch", type=int, default=C2["batch"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    cfg = {"workload": "C2: paged decode attention + KV append (Qwen2.5-1.5B attention shapes)",
           "layers": args.layers, "q_heads": C2["q_heads"], "kv_heads": C2["kv_heads"], "head_dim": C2["head_dim"],
           "block_size": C2["block_size"], "batch_per_gpu": args.batch, "global_batch": args.batch * world,
           "ctx": "U[{},{}] seeded per rank".format(C2["ctx_lo"], C2["ctx_hi"]),
           "block_tables": "random permutation of a pool holding every context",
           "l2": "no flush needed: each attention launch reads ~151 MB of K/V (> 126 MB L2), layers disjoint",
           "parallelism": "dp{} (request-sharded, independent KV pools)".format(world)}

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
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000.0 * args.batch / value, 3),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": cfg, "impl": "reference",
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
                     "frac": round(achieved / hbm, 4), "traffic": None,
                     "kernel": "attn_tc_kernel + attn_combine_kernel (one paged decode attention op per layer)",
                     "algorithmic_bytes_per_launch": res["attn_bytes"], "ms_per_launch": round(res["attn_ms"], 5),
                     "peak_source": "{} (MEASURED_PEAKS.json hbm_gbs)".format(peak_kind)},
        "e2e": {"value": round(args.batch * world / (res["e2e_ms"] * 1e-3), 2), "unit": "tokens/s",
                "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"],
                "path": "public per-layer API (PagedKVCache.reserve/append/release + paged_attention), pinned host I/O"},
        "gpu_launches": res["launches"],
        "clocks": res["clocks"],
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
