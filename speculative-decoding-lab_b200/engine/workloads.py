"""Seeded synthetic workloads and model shapes of the benchmark configs C1-C5.

Pure Python + numpy (no torch, no package-relative imports) so the golden
fixture generator can load this file on its own.  No public dataset is
involved: every input is drawn from ``numpy.random.default_rng(seed)`` with
the shapes and distributions of the configs.
"""

from __future__ import annotations

from types import SimpleNamespace
from typing import Any, Dict, List, Tuple

import numpy as np

# name: transformers-style Qwen2 shape fields
QWEN_SHAPES: Dict[str, Dict[str, Any]] = {
    "c1-target": dict(hidden_size=256, num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
                      head_dim=64, intermediate_size=512, vocab_size=1024),
    "c1-draft": dict(hidden_size=256, num_hidden_layers=1, num_attention_heads=4, num_key_value_heads=2,
                     head_dim=64, intermediate_size=512, vocab_size=1024),
    "qwen2.5-0.5b": dict(hidden_size=896, num_hidden_layers=24, num_attention_heads=14, num_key_value_heads=2,
                         head_dim=64, intermediate_size=4864, vocab_size=151936),
    "qwen2.5-1.5b": dict(hidden_size=1536, num_hidden_layers=28, num_attention_heads=12, num_key_value_heads=2,
                         head_dim=128, intermediate_size=8960, vocab_size=151936),
    "qwen2.5-3b": dict(hidden_size=2048, num_hidden_layers=36, num_attention_heads=16, num_key_value_heads=2,
                       head_dim=128, intermediate_size=11008, vocab_size=151936),
}


def shape_config(name: str, rope_theta: float = 1e6, max_position_embeddings: int = 4096, **overrides: Any):
    """``SimpleNamespace`` config (Qwen2 field names) for one of QWEN_SHAPES."""
    cfg = dict(QWEN_SHAPES[name])
    cfg.update(rope_theta=rope_theta, max_position_embeddings=max_position_embeddings, rms_norm_eps=1e-6,
               attention_bias=True, tie_word_embeddings=False)
    cfg.update(overrides)
    return SimpleNamespace(**cfg)


# --------------------------------------------------------------------- C1
C1 = dict(num_requests=8, prompt_lo=16, prompt_hi=64, vocab=1024, gamma=4, max_new_tokens=32, block_size=16,
          weight_std=0.02, target_seed=1, draft_seed=2)


def c1_requests(seed: int = 0) -> List[Tuple[List[int], int, int]]:
    """8 requests: prompt length U[16,64], ids U[0,1024), 32 new tokens, all at step 0.

    Returns ``(prompt_ids, max_new_tokens, arrive_time)`` triples.
    """
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(C1["num_requests"]):
        n = int(rng.integers(C1["prompt_lo"], C1["prompt_hi"] + 1))
        ids = rng.integers(0, C1["vocab"], size=n).tolist()
        out.append(([int(x) for x in ids], C1["max_new_tokens"], 0))
    return out


def c1_uniforms(seed: int = 0, n: int = 1 << 16) -> np.ndarray:
    """The pre-drawn fp32 uniform stream of the C1 stochastic run."""
    rng = np.random.default_rng(10_000 + seed)
    return rng.random(n, dtype=np.float32)


# --------------------------------------------------------------------- C2
C2 = dict(num_layers=28, num_q_heads=12, num_kv_heads=2, head_dim=128, block_size=16, batch=64, ctx_lo=512,
          ctx_hi=4096)


def c2_layout(seed: int = 0, batch: int = 64, ctx_lo: int = 512, ctx_hi: int = 4096, block_size: int = 16):
    """Context lengths U[ctx_lo, ctx_hi] and block tables that are a random
    permutation of a pool holding exactly every context plus the appended token.

    Returns ``(ctx, tables, capacity)``; ``tables[b]`` covers ``ctx[b] + 1`` positions.
    """
    rng = np.random.default_rng(seed)
    ctx = rng.integers(ctx_lo, ctx_hi + 1, size=batch).astype(np.int64)
    nblk = (ctx + 1 + block_size - 1) // block_size
    capacity = int(nblk.sum())
    perm = rng.permutation(capacity).astype(np.int64)
    tables, o = [], 0
    for n in nblk:
        tables.append(perm[o:o + int(n)].tolist())
        o += int(n)
    return ctx.tolist(), tables, capacity


# --------------------------------------------------------------------- C3
C3 = dict(gamma=5, batch=32, ctx_lo=256, ctx_hi=2048, temperature=1.0, logit_std=2.0, vocab=151936,
          target="qwen2.5-1.5b", draft="qwen2.5-0.5b")

# --------------------------------------------------------------------- C4
C4 = dict(gamma=4, prompt_mu=6.0, prompt_sigma=0.8, prompt_cap=4096, out_lo=64, out_hi=512, arrival_rate=64.0,
          pool_fraction=0.8, temperature=1.0, vocab=151936, target="qwen2.5-1.5b", draft="qwen2.5-0.5b")


def c4_requests(seed: int = 0, n: int = 2048, mean_gap_steps: float = 1.0, vocab: int = 151936):
    """C4 requests: prompt length floor(lognormal(6, 0.8)) capped at 4096 (at
    least 1), ids U[0, vocab), output length U[64, 512], Poisson arrivals.

    The reference's scheduler clock is the step (one speculative round), so
    the arrival process is Poisson in steps with mean gap ``mean_gap_steps``
    (the caller maps the config's 64 requests/s per GPU onto rounds).
    Returns ``(prompt_ids, max_new_tokens, arrive_step)`` triples in arrival
    order.
    """
    c = C4
    rng = np.random.default_rng(seed)
    t = 0.0
    out = []
    for _ in range(n):
        length = int(min(c["prompt_cap"], max(1, np.floor(rng.lognormal(c["prompt_mu"], c["prompt_sigma"])))))
        ids = rng.integers(0, vocab, size=length)
        new = int(rng.integers(c["out_lo"], c["out_hi"] + 1))
        out.append(([int(x) for x in ids], new, int(t)))
        t += float(rng.exponential(mean_gap_steps))
    return out


def c4_requests_wall(seed: int = 0, n: int = 2048, rate_per_s: float = 64.0, vocab: int = 151936):
    """The C4 request stream with Poisson arrivals in seconds: the same draws
    as :func:`c4_requests` (prompt length, ids, output length, then the gap),
    with exponential gaps of mean ``1 / rate_per_s`` seconds.

    Returns ``(prompt_ids, max_new_tokens, arrive_seconds)`` triples in
    arrival order (the first at 0.0).
    """
    c = C4
    rng = np.random.default_rng(seed)
    t = 0.0
    out = []
    for _ in range(n):
        length = int(min(c["prompt_cap"], max(1, np.floor(rng.lognormal(c["prompt_mu"], c["prompt_sigma"])))))
        ids = rng.integers(0, vocab, size=length)
        new = int(rng.integers(c["out_lo"], c["out_hi"] + 1))
        out.append(([int(x) for x in ids], new, t))
        t += float(rng.exponential(1.0 / rate_per_s))
    return out


def c4_slices(requests, steps: int):
    """Cut an arrival-ordered request stream into ``steps`` consecutive
    slices of (nearly) equal size, each slice's arrival times rebased so its
    first request arrives at 0."""
    n = len(requests)
    out = []
    for k in range(steps):
        lo, hi = (k * n) // steps, ((k + 1) * n) // steps
        part = requests[lo:hi]
        t0 = part[0][2] if part else 0.0
        out.append([(ids, new, t - t0) for ids, new, t in part])
    return out


# --------------------------------------------------------------------- C5
C5 = dict(gamma=6, batch_per_gpu=16, ctx_lo=8192, ctx_hi=32768, temperature=0.8, new_tokens=256,
          target="qwen2.5-3b", draft="qwen2.5-1.5b")
