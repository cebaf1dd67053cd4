"""Logits-in sampling (sdl_sample_logits_rows, sdl_spec_sample_logits).

The logits-in kernels never write probability rows, but they derive every
p_i with the same canonical reduction as sdl_logits_to_probs, so their draws
must equal -- bit for bit -- the two-step path (probabilities, then
sdl_sample_rows / sdl_spec_sample), which the other sampler tests pin to the
oracle and the reference fixtures.  Equal means the same tokens, accept
lengths and uniform-stream consumption.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import sampler as osamp
from specdec.sampler import (
    UniformStream,
    probs_rows,
    sample_logits_rows,
    sample_rows,
    spec_sample,
    spec_sample_logits,
)

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _stream(us, start=0):
    s = UniformStream(DEV, uniforms=torch.from_numpy(us))
    if start:
        s.counter.fill_(start)
        s.reserve(start)
    return s


@pytest.mark.parametrize("V", [1, 5, 4096, 4097, 70000, 151936])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_sample_logits_rows_equals_probs_then_sample(V, dtype):
    g = torch.Generator().manual_seed(V)
    x = (torch.randn(24, V, generator=g) * 3.0).to(dtype)
    x[3, : V // 2] = float("-inf")  # a row with a masked half
    rng = np.random.default_rng(V)
    us = rng.random(64, dtype=np.float32)
    us[0], us[1] = 0.0, np.float32(1.0) - np.float32(2 ** -24)
    for T in (1.0, 0.7, 1e-3):
        xd = x.to(DEV)
        s1, s2 = _stream(us, 5), _stream(us, 5)
        want = sample_rows(probs_rows(xd, T, False), s1, offset=2)
        got = sample_logits_rows(xd, T, s2, offset=2)
        assert got.tolist() == want.tolist()


def test_probs_rows_canonical_matches_oracle_on_masked_rows():
    x = torch.randn(6, 9000) * 2.0
    x[1, :8999] = float("-inf")          # one finite logit: p is one-hot
    x[2, 4096:] = float("-inf")          # whole trailing chunks masked
    p = probs_rows(x.to(DEV), 0.9, False).cpu().numpy()
    ref = osamp.logits_to_probs(x.numpy(), 0.9)
    np.testing.assert_allclose(p, ref, rtol=2e-6, atol=1e-9)
    assert p[1, 8999] == 1.0 and float(p[1, :8999].max()) == 0.0


def _block(B, gamma, V, seed, spread, dtype):
    g = torch.Generator().manual_seed(seed)
    pl = torch.randn(B, gamma + 1, V, generator=g) * 2.0
    ql = pl[:, :gamma] + torch.randn(B, gamma, V, generator=g) * spread
    return pl.to(dtype).to(DEV), ql.to(dtype).to(DEV)


@pytest.mark.parametrize("B,gamma,V,spread", [(4, 4, 50, 0.2), (32, 5, 151936, 2.0), (16, 6, 9000, 0.5),
                                              (64, 4, 4096, 0.0), (3, 1, 10, 1.0), (128, 6, 600, 0.3)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_spec_sample_logits_equals_two_step_path(B, gamma, V, spread, dtype):
    pl, ql = _block(B, gamma, V, seed=B * 7 + gamma, spread=spread, dtype=dtype)
    T = 0.8
    q = probs_rows(ql.reshape(B * gamma, V), T, False).reshape(B, gamma, V)
    # proposals drawn from q (mostly accepted) mixed with arbitrary ids (mostly rejected)
    us0 = np.random.default_rng(B).random(B * gamma, dtype=np.float32)
    draws = sample_rows(q.reshape(B * gamma, V), _stream(us0)).reshape(B, gamma)
    rnd = torch.randint(0, V, (B, gamma), generator=torch.Generator().manual_seed(3)).to(DEV, torch.int32)
    props = torch.where(torch.arange(gamma, device=DEV)[None, :] % 3 == 2, rnd, draws).contiguous()
    us = np.random.default_rng(B + 1).random(B * (gamma + 1) + 9, dtype=np.float32)
    p = probs_rows(pl.reshape(B * (gamma + 1), V), T, False).reshape(B, gamma + 1, V)
    s1, s2 = _stream(us, 2), _stream(us, 2)
    t1, n1 = spec_sample(p, q, props, s1, greedy=False, u_skip=3)
    t2, n2 = spec_sample_logits(pl, ql, T, props, s2, u_skip=3)
    n = n1.tolist()
    assert n2.tolist() == n
    a, b = t1.tolist(), t2.tolist()
    assert [a[i][: n[i]] for i in range(B)] == [b[i][: n[i]] for i in range(B)]
    assert s1.consumed() == s2.consumed()


def test_spec_sample_logits_residual_fallback_to_p():
    """q puts all mass where p has none at the proposal -> reject; the
    residual (p - q)+ then equals p everywhere except ... here p == q
    elsewhere, so the residual mass is 0 and the draw falls back to p."""
    V = 3
    pl = torch.tensor([[[0.0, float("-inf"), float("-inf")], [0.0, float("-inf"), float("-inf")]]], device=DEV)
    ql = torch.tensor([[[0.0, float("-inf"), float("-inf")]]], device=DEV)
    props = torch.tensor([[1]], dtype=torch.int32, device=DEV)  # q(1) = 0 and p(1) = 0 -> acceptance 0
    us = np.array([0.5, 0.25, 0.9], np.float32)
    s1, s2 = _stream(us), _stream(us)
    p = probs_rows(pl.reshape(2, V), 1.0, False).reshape(1, 2, V)
    q = probs_rows(ql.reshape(1, V), 1.0, False).reshape(1, 1, V)
    t1, n1 = spec_sample(p, q, props, s1, greedy=False)
    t2, n2 = spec_sample_logits(pl, ql, 1.0, props, s2)
    assert n2.tolist() == n1.tolist() == [1]
    assert t2[0, 0].item() == t1[0, 0].item() == 0
    assert s2.consumed() == s1.consumed() == 2


def test_spec_sample_logits_matches_oracle_softmax_path():
    """Against the oracle computing its own numpy softmax: same accept
    lengths and tokens on seeded blocks (no decision sits on a rounding
    boundary here)."""
    B, gamma, V = 8, 4, 2000
    pl, ql = _block(B, gamma, V, seed=11, spread=0.7, dtype=torch.float32)
    T = 1.0
    qn = osamp.logits_to_probs(ql.cpu().numpy(), T)
    pn = osamp.logits_to_probs(pl.cpu().numpy(), T)
    rng = np.random.default_rng(5)
    props = np.array([[osamp.sample_index(qn[b, j], rng.random(dtype=np.float32)) for j in range(gamma)]
                      for b in range(B)], np.int32)
    us = rng.random(B * (gamma + 1), dtype=np.float32)
    toks, n = spec_sample_logits(pl, ql, T, torch.from_numpy(props).to(DEV), _stream(us))
    want = osamp.batch_accept([pn[b] for b in range(B)], [[qn[b, j] for j in range(gamma)] for b in range(B)],
                              [props[b].tolist() for b in range(B)], osamp.UniformStream(us))
    nn, tk = n.tolist(), toks.tolist()
    assert [tk[b][: nn[b]] for b in range(B)] == want


def _set_mode(mode):
    from engine import _lib

    _lib.check(_lib.load().sdl_set_spec_sampler_mode(mode), "sdl_set_spec_sampler_mode")


@pytest.mark.parametrize("B,gamma,V,spread", [(32, 5, 151936, 2.0), (1, 1, 7, 0.3), (7, 4, 8193, 0.5),
                                              (100, 4, 151936, 1.0), (300, 4, 20000, 0.4), (700, 3, 5000, 0.4),
                                              (16, 32, 3000, 0.2)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_one_launch_sampler_equals_the_chain(B, gamma, V, spread, dtype):
    """sdl_spec_sample_logits' one-launch kernel (a cluster per sequence,
    the accept walk's uniform offsets found by waiting on lower sequences)
    against the five-launch chain: the same tokens, accept lengths and
    stream counter, on three consecutive rounds (the launch epoch moves on),
    with u_skip and a stream that does not start at 0.  Batches too large
    for one resident grid take the chain in both modes."""
    pl, ql = _block(B, gamma, V, seed=B + gamma, spread=spread, dtype=dtype)
    T = 0.9
    q = probs_rows(ql.reshape(B * gamma, V), T, False).reshape(B, gamma, V)
    us0 = np.random.default_rng(B + 5).random(B * gamma, dtype=np.float32)
    props = sample_rows(q.reshape(B * gamma, V), _stream(us0)).reshape(B, gamma).to(torch.int32).contiguous()
    us = np.random.default_rng(B + 6).random(3 * B * (gamma + 1) + 64, dtype=np.float32)
    results = []
    try:
        for mode in (0, 1):  # the chain, then the one-launch kernel
            _set_mode(mode)
            s = _stream(us, 3)
            rounds = []
            for _ in range(3):
                t, n = spec_sample_logits(pl, ql, T, props, s, u_skip=2)
                rounds.append((t.tolist(), n.tolist(), s.consumed()))
            results.append(rounds)
    finally:
        _set_mode(0)
    chain, fused = results
    for (t1, n1, c1), (t2, n2, c2) in zip(chain, fused):
        assert n1 == n2 and c1 == c2
        assert [t1[i][: n1[i]] for i in range(B)] == [t2[i][: n2[i]] for i in range(B)]
