"""Pin the numpy oracle to the reference's own outputs (CPU only).

Every fixture under tests/golden was produced by the reference
(tests/golden/make_golden.py); these tests replay the same inputs through
``oracle/`` and require identical integers (block tables, free lists, token
ids, accept lengths) and floats within the stated tolerances.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import load_json, load_npz
from oracle import attention as oatt
from oracle import kv as okv
from oracle import sampler as osamp


# ------------------------------------------------------------------ kv trace
def test_oracle_kv_trace_matches_reference():
    g = load_json("kv_trace.json")
    c = g["config"]
    kv = okv.PagedKVCache(c["num_layers"], c["num_kv_heads"], c["head_dim"], c["capacity"], c["block_size"])
    rng = np.random.default_rng(7)
    for step in g["ops"]:
        op = step["op"]
        if op[0] == "add":
            kv.add_sequence(op[1])
        elif op[0] == "write":
            vec = rng.standard_normal((2, 8)).astype(np.float32)
            kv.write(0, op[1], op[2], vec, vec)
        elif op[0] == "truncate":
            kv.truncate(op[1], op[2])
        elif op[0] == "clear":
            kv.clear(op[1])
        elif op[0] == "reset":
            kv.reset()
        st = step["state"]
        assert kv.block_tables == st["block_tables"], op
        assert kv.seq_lengths == st["seq_lengths"], op
        assert kv.num_allocated_blocks == st["num_allocated"], op
        assert kv.allocator.free_list() == st["free_list"], op


def test_oracle_exhaustion_message():
    g = load_json("kv_trace.json")
    kv = okv.PagedKVCache(1, 1, 8, 3, 4)
    kv.add_sequence(0)
    for pos in range(12):
        kv.write(0, 0, pos, np.zeros((1, 8), np.float32), np.zeros((1, 8), np.float32))
    with pytest.raises(okv.BlockExhaustedError) as e:
        kv.write(0, 0, 12, np.zeros((1, 8), np.float32), np.zeros((1, 8), np.float32))
    assert str(e.value) == g["exhaustion_message"]


# ----------------------------------------------------------------- attention
def _attn_case(a, tag):
    Hq, Hkv, d, bs, chunk, cap = (int(x) for x in a[tag + "_meta"])
    kv = okv.PagedKVCache(1, Hkv, d, cap, bs)
    kv.k[:] = a[tag + "_k"]
    kv.v[:] = a[tag + "_v"]
    tables = a[tag + "_tables"]
    starts = a[tag + "_starts"]
    for sid in range(len(starts)):
        kv.add_sequence(sid)
        kv.block_tables[sid] = [int(x) for x in tables[sid] if x >= 0]
        kv.seq_lengths[sid] = int(starts[sid]) + chunk
    q = a[tag + "_q"]
    if chunk == 1:
        out = oatt.paged_attention_decode(q[:, 0], kv, 0, range(len(starts)), starts + 1)[:, None]
    else:
        out = oatt.paged_attention_extend(q, kv, 0, range(len(starts)), starts)
    return out, a[tag + "_out"]


@pytest.mark.parametrize("tag", ["dec_f32_small", "dec_f32_d64", "ext_f32_d64"])
def test_oracle_attention_fp32_matches_reference(tag):
    """fp32: within 1e-5 relative (atol 1e-5) of the reference's SDPA."""
    out, ref = _attn_case(load_npz("attention.npz"), tag)
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("tag", ["dec_bf16_d128", "ext_bf16_d128", "dec_bf16_d64_r7"])
def test_oracle_attention_bf16_matches_reference(tag):
    """bf16: the reference output is bf16-rounded, so the exact (fp64) result
    must lie within one bf16 rounding step (2^-8 relative) plus 2e-3 * max|out|."""
    out, ref = _attn_case(load_npz("attention.npz"), tag)
    tol = 2.0 ** -8 * np.abs(out) + 2e-3 * np.abs(out).max()
    assert np.all(np.abs(out - ref) <= tol)


def test_oracle_prefill_chunk_matches_reference():
    a = load_npz("attention.npz")
    out = oatt.paged_attention_prefill_chunk(a["pre_f32_q"], a["pre_f32_k"], a["pre_f32_v"], a["pre_f32_lens"])
    np.testing.assert_allclose(out, a["pre_f32_out"], rtol=1e-5, atol=1e-5)
    assert np.all(out[0, 4:] == 0.0)


# ------------------------------------------------------------------- sampler
def test_oracle_logits_to_probs_matches_reference():
    for case in load_json("sampler.json")["probs"]:
        p = osamp.logits_to_probs(np.array(case["logits"], np.float32), case["T"])
        np.testing.assert_allclose(p, np.array(case["probs"]), rtol=1e-6, atol=1e-7)


def test_oracle_residual_matches_reference():
    for case in load_json("sampler.json")["residual"]:
        r = osamp.residual_distribution(np.array(case["p"], np.float32), np.array(case["q"], np.float32))
        np.testing.assert_allclose(r, np.array(case["residual"]), rtol=1e-6, atol=1e-8)


def test_oracle_draw_rule_matches_fixture():
    for case in load_json("sampler.json")["draw"]:
        w = np.array(case["w"], np.float32)
        got = [osamp.sample_index(w, np.float32(u)) for u in case["u"]]
        assert got == case["idx"]


def test_oracle_batch_accept_kats():
    for case in load_json("sampler.json")["accept_kat"]:
        sids = list(case["p"].keys())
        p = [np.array(case["p"][s], np.float32) for s in sids]
        q = [[np.array(r, np.float32) for r in case["q"][s]] for s in sids]
        props = [case["proposals"][s] for s in sids]
        acc = osamp.batch_accept(p, q, props, osamp.UniformStream(case["u"]))
        assert {s: a for s, a in zip(sids, acc)} == case["accepted"]


def test_oracle_batch_accept_stochastic_matches_reference():
    for case in load_json("sampler.json")["accept_stoch"]:
        pl = np.array(case["p_logits"], np.float32)
        ql = np.array(case["q_logits"], np.float32)
        T = case["T"]
        B, gp1, _ = pl.shape
        p = [osamp.logits_to_probs(pl[b], T) for b in range(B)]
        q = [[osamp.logits_to_probs(ql[b, j], T) for j in range(gp1 - 1)] for b in range(B)]
        props = [case["proposals"][str(b)] for b in range(B)]
        acc = osamp.batch_accept(p, q, props, osamp.UniformStream(case["u"]))
        assert acc == [case["accepted"][str(b)] for b in range(B)]


def test_fp32_weight_rule_equals_double_rule():
    """The kernels compute W = floor(w * 2^62) as the fp32 product with 2^62
    (exact: a power-of-two scaling) truncated to u64 with saturation
    (csrc/sampler*.cu wfix).  The premise -- the fp32 product equals the
    exact product wherever it is below 2^64 -- and the resulting integers
    must match the oracle's double-precision floor on edge and random values."""
    vals = [0.0, -1.0, float("nan"), float("inf"), 1e-45, 2.0 ** -62, 2.0 ** -62 * 1.5, 2.0 ** -63, 2.0 ** -40,
            0.5, 1.0, 1.9999999, 2.0, 3.9999998, 4.0, 7.5]
    rng = np.random.default_rng(0)
    vals += list(rng.random(2000).astype(np.float32)) + list((rng.random(500) * 1e-12).astype(np.float32))
    w = np.array(vals, dtype=np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        prod32 = w * np.float32(2.0 ** 62)                       # what the kernel multiplies
        exact = w.astype(np.float64) * 2.0 ** 62
    finite = np.isfinite(exact) & (exact < 2.0 ** 64)
    assert np.array_equal(prod32[finite].astype(np.float64), exact[finite])

    def trunc_sat(x: float) -> int:                              # cvt.rzi.u64.f32 semantics
        if x != x or x <= 0.0:
            return 0
        if x >= 2.0 ** 64:
            return (1 << 64) - 1
        return int(x)

    want = [int(v) for v in osamp.wfix(w)]
    assert [trunc_sat(float(x)) for x in prod32] == want
