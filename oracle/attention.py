"""Oracle attention: restates engine/attention.py:32-215 in numpy (fp64 math).

Test infrastructure only (see oracle/__init__.py).
"""

from __future__ import annotations

from typing import Sequence

import numpy as np

from .kv import PagedKVCache


def expand_to_q_heads(x: np.ndarray, num_q_heads: int) -> np.ndarray:
    """repeat_interleave over the head axis (engine/attention.py:32-38)."""
    ratio = num_q_heads // x.shape[-2]
    return x if ratio == 1 else np.repeat(x, ratio, axis=-2)


def attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, limits: Sequence[int]) -> np.ndarray:
    """Rows of ``q`` (rows, Hq, d) attend ``k/v`` (L, Hkv, d); row r sees [0, limits[r]).

    Scale 1/sqrt(d) like SDPA's default (engine/attention.py:92,212); q head h
    reads kv head h // (Hq/Hkv) (engine/attention.py:32-38).  fp64 matmuls per
    kv head (BLAS releases the GIL, so callers may thread over sequences).
    """
    rows, Hq, d = q.shape
    L, Hkv = k.shape[0], k.shape[1]
    ratio = Hq // Hkv
    scale = 1.0 / np.sqrt(d)
    mask = np.arange(L)[None, :] < np.asarray(limits)[:, None]  # (rows, L)
    out = np.empty((rows, Hq, d), dtype=np.float64)
    q64 = q.astype(np.float64)
    for g in range(Hkv):
        kg = k[:, g, :].astype(np.float64)
        vg = v[:, g, :].astype(np.float64)
        qg = q64[:, g * ratio:(g + 1) * ratio, :].reshape(rows * ratio, d)
        s = (qg @ kg.T) * scale                                   # (rows*ratio, L)
        s = np.where(np.repeat(mask, ratio, axis=0), s, -np.inf)
        s -= s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=-1, keepdims=True)
        out[:, g * ratio:(g + 1) * ratio, :] = (p @ vg).reshape(rows, ratio, d)
    return out


def paged_attention_decode(q2d: np.ndarray, kv: PagedKVCache, layer: int, seq_ids, lengths) -> np.ndarray:
    """engine/attention.py:96-118: row b attends its first lengths[b] positions."""
    out = np.zeros(q2d.shape, dtype=np.float64)
    for b, (sid, ln) in enumerate(zip(seq_ids, lengths)):
        k, v = kv.gather(layer, sid, int(ln))
        out[b] = attend(q2d[b][None], k, v, [int(ln)])[0]
    return out


def paged_attention_extend(q3d: np.ndarray, kv: PagedKVCache, layer: int, seq_ids, starts) -> np.ndarray:
    """engine/attention.py:170-215: row j attends 0..start+j inclusive."""
    B, chunk = q3d.shape[:2]
    out = np.zeros(q3d.shape, dtype=np.float64)
    for b, (sid, st) in enumerate(zip(seq_ids, starts)):
        st = int(st)
        k, v = kv.gather(layer, sid, st + chunk)
        out[b] = attend(q3d[b], k, v, [st + j + 1 for j in range(chunk)])
    return out


def paged_attention_prefill_chunk(q3d: np.ndarray, k3d: np.ndarray, v3d: np.ndarray, lengths) -> np.ndarray:
    """engine/attention.py:121-167: causal within the chunk, padded rows zero."""
    out = np.zeros(q3d.shape, dtype=np.float64)
    for b, ln in enumerate(lengths):
        ln = int(ln)
        if ln <= 0:
            continue
        out[b, :ln] = attend(q3d[b, :ln], k3d[b, :ln], v3d[b, :ln], [j + 1 for j in range(ln)])
    return out
