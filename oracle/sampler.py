"""Oracle sampling math: restates specdec/sampler.py:19-92 and
engine/spec_scheduler.py:41-88 in numpy, plus the defined draw rule.

Test infrastructure only (see oracle/__init__.py).

Defined inverse-CDF draw (shared with the sdl_sample_rows kernel): weights w
(fp32, any scale with sum < 4), uniform u (fp32 in [0, 1)):
    W_i = floor(w_i * 2^62), S = sum W_i, U = floor(u * 2^64),
    target = floor(U * S / 2^64), token = min{ i : W_0 + ... + W_i > target }.
It stands in for torch.multinomial (specdec/sampler.py:66-69), whose internal
draw cannot be reproduced; given the same uniform both sides pick the same id.
"""

from __future__ import annotations

from typing import List, Sequence

import numpy as np

EPS = 1e-12
_TWO62 = float(2 ** 62)
_TWO64 = float(2 ** 64)
_U64MAX = np.uint64(0xFFFFFFFFFFFFFFFF)


class UniformStream:
    """Pre-drawn fp32 uniforms consumed in order."""

    def __init__(self, values) -> None:
        self.values = np.asarray(values, dtype=np.float32).reshape(-1)
        self.pos = 0

    def next(self) -> np.float32:
        if self.pos >= self.values.size:
            raise RuntimeError("uniform stream exhausted")
        u = self.values[self.pos]
        self.pos += 1
        return u


def wfix(w: np.ndarray) -> np.ndarray:
    x = np.asarray(w, dtype=np.float32).astype(np.float64)
    x = np.where(x > 0, x, 0.0) * _TWO62
    big = x >= _TWO64
    out = np.floor(np.where(big, 0.0, x)).astype(np.uint64)
    out[big] = _U64MAX
    return out


def ufix(u) -> int:
    u = float(np.float32(u))
    if not u > 0:
        return 0
    x = u * _TWO64
    return (1 << 64) - 1 if x >= _TWO64 else int(x)


def weight_sum(w: np.ndarray) -> int:
    return int(wfix(w).sum(dtype=np.uint64))


def sample_index(w: np.ndarray, u) -> int:
    W = wfix(np.asarray(w).reshape(-1))
    c = np.cumsum(W, dtype=np.uint64)
    S = int(c[-1])
    if S == 0:
        raise ValueError("invalid multinomial distribution (sum of probabilities <= 0)")
    target = (ufix(u) * S) >> 64
    return int(np.searchsorted(c, np.uint64(target), side="right"))


def logits_to_probs(logits: np.ndarray, temperature: float, top_k: int = 0, top_p: float = 1.0,
                    eps: float = EPS) -> np.ndarray:
    """specdec/sampler.py:19-36 in fp32 (greedy: one-hot at the first argmax)."""
    x = np.asarray(logits, dtype=np.float32)
    if temperature <= 0.0:
        out = np.zeros_like(x)
        idx = np.argmax(x, axis=-1)
        np.put_along_axis(out, idx[..., None], np.float32(1.0), axis=-1)
        return out
    scaled = x / np.float32(max(temperature, eps))
    scaled = apply_top_k(scaled, top_k)
    scaled = apply_top_p(scaled, top_p)
    m = scaled.max(axis=-1, keepdims=True)
    e = np.exp(scaled - m).astype(np.float32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


def apply_top_k(x: np.ndarray, top_k: int) -> np.ndarray:
    if top_k <= 0 or top_k >= x.shape[-1]:
        return x
    kth = -np.sort(-x, axis=-1)[..., top_k - 1: top_k]
    return np.where(x < kth, np.float32(-np.inf), x)


def apply_top_p(x: np.ndarray, top_p: float) -> np.ndarray:
    if top_p >= 1.0 or top_p <= 0.0:
        return x
    order = np.argsort(-x, axis=-1, kind="stable")
    sx = np.take_along_axis(x, order, axis=-1)
    e = np.exp(sx - sx.max(axis=-1, keepdims=True))
    sm = e / e.sum(axis=-1, keepdims=True)
    mask = np.cumsum(sm, axis=-1) - sm >= top_p
    sx = np.where(mask, np.float32(-np.inf), sx)
    out = np.empty_like(x)
    np.put_along_axis(out, order, sx, axis=-1)
    return out


def acceptance_probability(p: np.ndarray, q: np.ndarray, token_id: int) -> float:
    """specdec/sampler.py:86-92 (Python floats, i.e. fp64)."""
    q_prob = float(q[token_id])
    p_prob = float(p[token_id])
    if q_prob <= EPS:
        return 1.0 if p_prob > EPS else 0.0
    return float(min(1.0, p_prob / q_prob))


def residual_weights(p: np.ndarray, q: np.ndarray) -> np.ndarray:
    """clamp(p - q, 0) in fp32 (specdec/sampler.py:78)."""
    return np.maximum(np.asarray(p, np.float32) - np.asarray(q, np.float32), np.float32(0.0))


def residual_distribution(p: np.ndarray, q: np.ndarray) -> np.ndarray:
    """specdec/sampler.py:72-83 (normalised)."""
    r = residual_weights(p, q)
    total = r.sum(dtype=np.float32)
    if float(total) <= EPS:
        return (p / max(float(np.sum(p, dtype=np.float32)), EPS)).astype(np.float32)
    return (r / total).astype(np.float32)


def residual_draw(p: np.ndarray, q: np.ndarray, u) -> int:
    """The rejection draw: (p - q)+ unless its mass is <= 1e-12, then p."""
    r = residual_weights(p, q)
    if weight_sum(r) / _TWO62 <= EPS:
        return sample_index(p, u)
    return sample_index(r, u)


def batch_accept(p_rows: Sequence[np.ndarray], q_rows: Sequence[Sequence[np.ndarray]],
                 proposals: Sequence[Sequence[int]], stream: UniformStream) -> List[List[int]]:
    """engine/spec_scheduler.py:46-88 with every uniform taken from ``stream``."""
    out: List[List[int]] = []
    for p_all, q_list, props in zip(p_rows, q_rows, proposals):
        gamma = len(props)
        accepted: List[int] = []
        rejected = False
        for j in range(gamma):
            x = int(props[j])
            u = stream.next()
            if float(u) < acceptance_probability(p_all[j], q_list[j], x):
                accepted.append(x)
            else:
                accepted.append(residual_draw(p_all[j], q_list[j], stream.next()))
                rejected = True
                break
        if not rejected:
            accepted.append(sample_index(p_all[gamma], stream.next()))
        out.append(accepted)
    return out
