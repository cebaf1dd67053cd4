"""Paged attention at the long-context config's key spans (16k-32k keys).

The C5 config runs the 7-row verify (gamma = 6) of a Qwen2.5-3B-shaped target
(16 q heads, 2 kv heads, head_dim 128) and 1.5B-shaped draft decodes (12 q
heads) over contexts U[8192, 32768].  Every launch plan -- the automatic
choice, the persistent tcgen05 kernel, mma.sync with keys or query rows on
the MMA M dimension, register-direct loads, the CUDA-core kernel, explicit
split sizes and the on-chip cluster merge -- is checked here against the
fp64 oracle (engine/attention.py:96-118 and 170-215 restated) at spans of
16,384 to 32,767 keys, where the split-K plans reach hundreds of splits per
row and the online softmax rescales many times.

Tolerances: ``conftest.check_attention_16bit`` (per element on the fp32
output, normwise and one bf16 rounding on the 16-bit output).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import check_attention_16bit
from engine.attention import AttnBatch, attention_kernel, paged_attention
from oracle import attention as oatt
from test_attention_gpu import _build

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)

GAMMA = 6
CHUNK = GAMMA + 1
STARTS = [16384, 24000, 32760]          # verify rows j attend start + j + 1 keys
DECODE_STARTS = [16390, 24006, 32766]   # decode rows attend start + 1 keys (sequence b holds STARTS[b] + 7)


@pytest.fixture(scope="module")
def long_cache():
    """One cache holding the three sequences (scattered block tables)."""
    kv, ref = _build([s + CHUNK for s in STARTS], 2, 128, 16, torch.bfloat16, seed=77, piece=200)
    return kv, ref


def _exact(q, ref, starts):
    return oatt.paged_attention_extend(q.float().cpu().numpy(), ref, 0, range(len(starts)), starts)


# (use_umma, mma_layout, force_generic, pages_per_split, cluster_merge)
VERIFY_PLANS = [
    (0, 0, False, 0, False),    # automatic
    (1, 0, False, 0, False),    # persistent tcgen05 (stream-K slot merge)
    (1, 0, False, 12, False),   # tcgen05 with 192-key splits (tiles end inside a split)
    (-1, 1, False, 0, False),   # mma.sync, keys on M (TMA ring)
    (-1, 1, False, 3, False),   # ... 48-key splits: 680+ splits per row
    (-1, 1, False, 64, True),   # ... 1024-key splits merged on chip in a cluster
    (-1, 2, False, 0, False),   # mma.sync, query rows on M
    (-1, 2, False, 12, False),
    (-1, 3, False, 0, False),   # register-direct loads
    (0, 0, True, 0, False),     # CUDA-core kernel
]


@pytest.mark.parametrize("plan", range(len(VERIFY_PLANS)))
def test_c5_verify_spans_match_oracle(long_cache, plan):
    """7-row verify at 16k-32k keys, ratio 8 (C5 target shape), every plan."""
    kv, ref = long_cache
    umma, layout, generic, pps, cluster = VERIFY_PLANS[plan]
    g = torch.Generator().manual_seed(1000 + plan)
    q = torch.randn(len(STARTS), CHUNK, 16, 128, generator=g).to(DEV, torch.bfloat16)
    batch = AttnBatch.from_lists(DEV, list(range(len(STARTS))), STARTS, CHUNK)
    kw = dict(use_umma=umma, mma_layout=layout, force_generic=generic, pages_per_split=pps, cluster_merge=cluster)
    out = paged_attention(q, kv, 0, batch, **kw)
    out32 = paged_attention(q, kv, 0, batch, out_dtype=torch.float32, **kw)
    check_attention_16bit(out.float().cpu().numpy(), out32.cpu().numpy(), _exact(q, ref, STARTS))
    kv.check_errors()


DECODE_PLANS = [
    (0, 0, False, 0, False),    # automatic
    (-1, 1, False, 0, False),   # attn_tc_kernel (keys on M, TMA ring)
    (-1, 1, False, 4, False),
    (-1, 1, False, 64, True),
    (-1, 3, False, 0, False),   # register-direct
    (-1, 2, False, 0, False),   # query rows on M
    (1, 0, False, 0, False),    # tcgen05
    (0, 0, True, 0, False),     # CUDA-core kernel
]


@pytest.mark.parametrize("plan", range(len(DECODE_PLANS)))
@pytest.mark.parametrize("hq", [12, 16])
def test_decode_at_32k_keys_matches_oracle(long_cache, plan, hq):
    """Decode rows of 16,391-32,767 keys (C5 draft decode at ratio 6, and
    ratio 8) on every plan."""
    kv, ref = long_cache
    umma, layout, generic, pps, cluster = DECODE_PLANS[plan]
    g = torch.Generator().manual_seed(2000 + plan + hq)
    q = torch.randn(len(DECODE_STARTS), 1, hq, 128, generator=g).to(DEV, torch.bfloat16)
    batch = AttnBatch.from_lists(DEV, list(range(len(DECODE_STARTS))), DECODE_STARTS, 1)
    kw = dict(use_umma=umma, mma_layout=layout, force_generic=generic, pages_per_split=pps, cluster_merge=cluster)
    out = paged_attention(q, kv, 0, batch, **kw)
    out32 = paged_attention(q, kv, 0, batch, out_dtype=torch.float32, **kw)
    check_attention_16bit(out.float().cpu().numpy(), out32.cpu().numpy(), _exact(q, ref, DECODE_STARTS))
    kv.check_errors()


def test_automatic_plans_at_c5_spans_are_the_fast_kernels(long_cache):
    """The automatic choice at these spans is a tensor-core kernel, not the
    CUDA-core fallback (the parity above covers whichever it is)."""
    kv, _ = long_cache
    qv = torch.zeros(len(STARTS), CHUNK, 16, 128, device=DEV, dtype=torch.bfloat16)
    qd = torch.zeros(len(DECODE_STARTS), 1, 12, 128, device=DEV, dtype=torch.bfloat16)
    kv_ = attention_kernel(qv, kv, AttnBatch.from_lists(DEV, [0, 1, 2], STARTS, CHUNK))
    kd_ = attention_kernel(qd, kv, AttnBatch.from_lists(DEV, [0, 1, 2], DECODE_STARTS, 1))
    assert kv_ != "generic" and kd_ != "generic"


def test_long_span_results_are_deterministic(long_cache):
    """Repeated calls at 32k keys give identical bits (fixed split sizes and
    a fixed merge order)."""
    kv, _ = long_cache
    q = torch.randn(len(STARTS), CHUNK, 16, 128, device=DEV, dtype=torch.bfloat16)
    batch = AttnBatch.from_lists(DEV, [0, 1, 2], STARTS, CHUNK)
    first = paged_attention(q, kv, 0, batch)
    for _ in range(3):
        assert torch.equal(paged_attention(q, kv, 0, batch), first)
