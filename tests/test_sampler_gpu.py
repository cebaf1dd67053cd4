"""Sampling kernels vs the reference fixtures and the oracle.

Integer work is bit-exact: argmax indices, inverse-CDF draws given the same
uniforms, accept lengths and accepted tokens, uniform-stream consumption.
Probabilities are fp32 softmax: within 1e-6 relative of the reference.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_json
from engine.spec_scheduler import batch_accept
from oracle import sampler as osamp
from specdec.config import SamplingConfig
from specdec.sampler import (
    UniformStream,
    argmax_rows,
    logits_to_probs,
    probs_rows,
    residual_distribution,
    sample_rows,
    sample_token,
    spec_sample,
)

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_logits_to_probs_matches_reference_fixture():
    for case in load_json("sampler.json")["probs"]:
        logits = torch.tensor(case["logits"], device=DEV)
        p = logits_to_probs(logits, SamplingConfig(temperature=case["T"]))
        np.testing.assert_allclose(p.cpu().numpy(), np.array(case["probs"]), rtol=1e-6, atol=1e-7)


def test_greedy_one_hot_and_argmax_first_index_on_ties():
    x = torch.tensor([[0.1, 2.0, -1.0, 2.0], [5.0, 5.0, 5.0, 5.0]], device=DEV)
    assert argmax_rows(x).tolist() == [1, 0]
    p = logits_to_probs(x, SamplingConfig(temperature=0.0))
    assert p.tolist() == [[0, 1, 0, 0], [1, 0, 0, 0]]


def test_top_k_top_p_filtering():
    logits = torch.tensor([[5.0, 4.0, 3.0, 2.0, 1.0]], device=DEV)
    p = logits_to_probs(logits, SamplingConfig(temperature=1.0, top_k=2))
    assert int((p > 0).sum()) == 2
    logits = torch.log(torch.tensor([[0.5, 0.3, 0.15, 0.05]], device=DEV))
    p = logits_to_probs(logits, SamplingConfig(temperature=1.0, top_p=0.8))
    assert float(p[0, 3]) == 0.0 and float(p.sum()) >= 0.8 - 1e-6


@pytest.mark.parametrize("V", [7, 1000, 151936])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_probs_kernel_matches_oracle(V, dtype):
    logits = (torch.randn(5, V, device=DEV) * 2.0).to(dtype)
    for T in (1.0, 0.8):
        p = probs_rows(logits, T, False).cpu().numpy()
        ref = osamp.logits_to_probs(logits.float().cpu().numpy(), T)
        np.testing.assert_allclose(p, ref, rtol=2e-6, atol=1e-9)


def test_draw_rule_matches_fixture_and_oracle_exactly():
    for case in load_json("sampler.json")["draw"]:
        w = torch.tensor(case["w"], dtype=torch.float32, device=DEV)
        us = np.array(case["u"], np.float32)
        stream = UniformStream(DEV, uniforms=torch.from_numpy(us))
        got = sample_rows(w.unsqueeze(0).expand(len(us), -1).contiguous(), stream).tolist()
        assert got == case["idx"]
    rng = np.random.default_rng(4)
    for V in (3, 64, 5000, 151936):
        for spiky in (False, True):
            x = rng.standard_normal((16, V)).astype(np.float32) * (8.0 if spiky else 1.0)
            w = osamp.logits_to_probs(x, 1.0)
            us = rng.random(16, dtype=np.float32)
            us[0] = 0.0
            us[1] = np.float32(1.0) - np.float32(2 ** -24)
            stream = UniformStream(DEV, uniforms=torch.from_numpy(us))
            got = sample_rows(torch.from_numpy(w).to(DEV), stream).tolist()
            assert got == [osamp.sample_index(w[r], us[r]) for r in range(16)]


def test_sample_token_and_residual_api():
    p = torch.tensor([0.5, 0.3, 0.2], device=DEV)
    q = torch.tensor([0.1, 0.4, 0.5], device=DEV)
    r = residual_distribution(p, q)
    assert abs(float(r.sum()) - 1.0) < 1e-6 and float(r[2]) == 0.0
    s = UniformStream(DEV, uniforms=torch.tensor([0.0, 0.6, 0.99]))
    assert [sample_token(p, s) for _ in range(3)] == [0, 1, 2]
    assert s.consumed() == 3


def _random_block(B, gamma, V, T, seed, spread):
    g = torch.Generator(device="cpu").manual_seed(seed)
    pl = torch.randn(B, gamma + 1, V, generator=g) * 2.0
    ql = pl[:, :gamma] + torch.randn(B, gamma, V, generator=g) * spread
    p = probs_rows(pl.to(DEV), T, False).reshape(B, gamma + 1, V)
    q = probs_rows(ql.to(DEV), T, False).reshape(B, gamma, V)
    props = torch.stack([torch.argmax(q[:, j], -1) if j % 2 == 0 else
                         torch.randint(0, V, (B,), generator=g).to(DEV) for j in range(gamma)], 1).to(torch.int32)
    return p, q, props


@pytest.mark.parametrize("B,gamma,V,spread", [(4, 4, 50, 0.2), (32, 5, 151936, 1.0), (16, 6, 3000, 3.0),
                                              (128, 6, 600, 0.5), (3, 1, 10, 0.0)])
def test_spec_sample_matches_oracle_batch_accept(B, gamma, V, spread):
    p, q, props = _random_block(B, gamma, V, 1.0, seed=B * 31 + gamma, spread=spread)
    us = np.random.default_rng(B).random(B * (gamma + 1) + 7, dtype=np.float32)
    stream = UniformStream(DEV, uniforms=torch.from_numpy(us))
    stream.counter.fill_(3)
    stream.reserve(3)
    tokens, n_out = spec_sample(p, q, props, stream, greedy=False, u_skip=4)
    pn, qn, pr = p.cpu().numpy(), q.cpu().numpy(), props.cpu().numpy()
    ostream = osamp.UniformStream(us)
    ostream.pos = 7
    want = osamp.batch_accept([pn[b] for b in range(B)], [[qn[b, j] for j in range(gamma)] for b in range(B)],
                              [pr[b].tolist() for b in range(B)], ostream)
    n = n_out.tolist()
    tk = tokens.tolist()
    assert [tk[b][: n[b]] for b in range(B)] == want
    assert stream.consumed() == ostream.pos


def test_spec_sample_greedy_rule():
    B, gamma, V = 6, 4, 40
    g = torch.Generator().manual_seed(1)
    pl = torch.randn(B, gamma + 1, V, generator=g).to(DEV)
    p_arg = argmax_rows(pl.reshape(-1, V)).reshape(B, gamma + 1)
    props = p_arg[:, :gamma].clone()
    props[1, 0] = (props[1, 0] + 1) % V
    props[3, 2] = (props[3, 2] + 1) % V
    tokens, n_out = spec_sample(None, None, props, None, greedy=True, p_arg=p_arg)
    pa = p_arg.tolist()
    for b in range(B):
        n = n_out[b].item()
        row = tokens[b, :n].tolist()
        if b == 1:
            assert row == [pa[1][0]]
        elif b == 3:
            assert row == pa[3][:3]
        else:
            assert row == pa[b]


def test_batch_accept_reference_kats():
    for case in load_json("sampler.json")["accept_kat"]:
        p_by = {int(k): torch.tensor(v, device=DEV) for k, v in case["p"].items()}
        q_by = {int(k): [torch.tensor(r, device=DEV) for r in v] for k, v in case["q"].items()}
        prop = {int(k): v for k, v in case["proposals"].items()}
        acc = batch_accept(p_by, q_by, prop, UniformStream(DEV, uniforms=torch.tensor(case["u"])))
        assert {str(k): v for k, v in acc.items()} == case["accepted"]


def test_batch_accept_reference_stochastic_cases():
    """Reference probabilities recomputed by our kernel from the same logits;
    identical accepted tokens given the same uniform stream."""
    for case in load_json("sampler.json")["accept_stoch"]:
        pl = torch.tensor(case["p_logits"], device=DEV)
        ql = torch.tensor(case["q_logits"], device=DEV)
        sc = SamplingConfig(temperature=case["T"])
        B, gp1, V = pl.shape
        p_by = {b: logits_to_probs(pl[b], sc) for b in range(B)}
        q_by = {b: [logits_to_probs(ql[b, j], sc) for j in range(gp1 - 1)] for b in range(B)}
        prop = {b: case["proposals"][str(b)] for b in range(B)}
        acc = batch_accept(p_by, q_by, prop, UniformStream(DEV, uniforms=torch.tensor(case["u"])))
        assert {str(k): v for k, v in acc.items()} == case["accepted"]
