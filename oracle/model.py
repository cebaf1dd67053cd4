"""Oracle decoder forward in numpy over the oracle paged cache.

Restates the per-layer computation of engine/model.py:123-194,369-398 (toy)
and engine/qwen.py:100-199 (Qwen2, q/k/v biases) in fp32, attention in fp64
(oracle.attention).  Test infrastructure only (see oracle/__init__.py).
"""

from __future__ import annotations

from typing import Dict, Optional, Sequence

import numpy as np

from .attention import attend
from .kv import PagedKVCache


def rotary_table(head_dim: int, theta: float, max_len: int) -> np.ndarray:
    """(max_len, 2, head_dim) cos/sin, rotate_half layout (engine/model.py:41-53)."""
    inv_freq = (1.0 / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.float32) / np.float32(head_dim))))
    inv_freq = inv_freq.astype(np.float32)
    pos = np.arange(max_len, dtype=np.float32)[:, None]
    freqs = (pos * inv_freq[None, :]).astype(np.float32)
    emb = np.concatenate((freqs, freqs), axis=-1)
    return np.stack((np.cos(emb), np.sin(emb)), axis=1).astype(np.float32)


def _rotate_half(x: np.ndarray) -> np.ndarray:
    d = x.shape[-1]
    return np.concatenate((-x[..., d // 2:], x[..., : d // 2]), axis=-1)


def _rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    return (x * cos + _rotate_half(x) * sin).astype(np.float32)


def _rms(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    rms = np.sqrt(np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps))
    return ((x / rms) * w).astype(np.float32)


class NumpyPagedLM:
    """A Qwen2-style (``kind='qwen'``) or toy (``kind='toy'``) decoder.

    ``params`` uses the torch state-dict names of the corresponding model.
    """

    def __init__(self, params: Dict[str, np.ndarray], num_layers: int, num_q_heads: int, num_kv_heads: int,
                 head_dim: int, rope: np.ndarray, kind: str = "qwen", eps: float = 1e-6) -> None:
        self.p = {k: np.asarray(v, dtype=np.float32) for k, v in params.items()}
        self.num_layers = num_layers
        self.nq = num_q_heads
        self.nkv = num_kv_heads
        self.d = head_dim
        self.rope = rope.astype(np.float32)
        self.kind = kind
        self.eps = eps
        self.vocab_size = self.p["lm_head.weight"].shape[0]

    def _lin(self, x: np.ndarray, name: str) -> np.ndarray:
        y = x @ self.p[name + ".weight"].T
        b = self.p.get(name + ".bias")
        if b is not None:
            y = y + b
        return y.astype(np.float32)

    def _names(self, i: int):
        if self.kind == "qwen":
            a = "layers.{}.self_attn.".format(i)
            m = "layers.{}.mlp.".format(i)
            return a + "q_proj", a + "k_proj", a + "v_proj", a + "o_proj", m + "gate_proj", m + "up_proj", m + "down_proj"
        a = "layers.{}.".format(i)
        return a + "q", a + "k", a + "v", a + "o", a + "mlp.gate", a + "mlp.up", a + "mlp.down"

    def _mlp(self, x: np.ndarray, g: str, u: str, dn: str) -> np.ndarray:
        gate = self._lin(x, g)
        silu = (gate / (np.float32(1.0) + np.exp(-gate))).astype(np.float32)
        return self._lin((silu * self._lin(x, u)).astype(np.float32), dn)

    def _logits(self, h: np.ndarray) -> np.ndarray:
        return self._lin(_rms(h, self.p["norm.weight"], self.eps), "lm_head")

    def _layer(self, i: int, h: np.ndarray, positions: np.ndarray, attend_fn) -> np.ndarray:
        """h: (T, H) rows at ``positions``; attend_fn(i, q, k, v) -> (T, Hq, d)."""
        qn, kn, vn, on, gn, un, dn = self._names(i)
        x = _rms(h, self.p["layers.{}.input_layernorm.weight".format(i)], self.eps)
        T = h.shape[0]
        cos = self.rope[positions, 0][:, None, :]
        sin = self.rope[positions, 1][:, None, :]
        q = _rope(self._lin(x, qn).reshape(T, self.nq, self.d), cos, sin)
        k = _rope(self._lin(x, kn).reshape(T, self.nkv, self.d), cos, sin)
        v = self._lin(x, vn).reshape(T, self.nkv, self.d)
        out = attend_fn(i, q, k, v).astype(np.float32)
        h = (h + self._lin(out.reshape(T, -1), on)).astype(np.float32)
        return (h + self._mlp(_rms(h, self.p["layers.{}.post_attention_layernorm.weight".format(i)], self.eps),
                              gn, un, dn)).astype(np.float32)

    def _embed(self, ids) -> np.ndarray:
        return self.p["embed_tokens.weight"][np.asarray(ids, dtype=np.int64)].astype(np.float32)

    def prefill(self, ids: Sequence[int], kv: PagedKVCache, sid: int) -> np.ndarray:
        """One prompt: causal attention within it, then K/V written (engine/qwen.py:171-199)."""
        P = len(ids)
        h = self._embed(ids)
        pos = np.arange(P)

        def fn(i, q, k, v):
            out = attend(q, k, v, [j + 1 for j in range(P)])
            for t in range(P):
                kv.write(i, sid, t, k[t], v[t])
            return out

        for i in range(self.num_layers):
            h = self._layer(i, h, pos, fn)
        return self._logits(h[-1:])[0]

    def forward_rows(self, ids_2d: np.ndarray, kv: PagedKVCache, seq_ids: Sequence[int],
                     starts: Sequence[int], slots: Optional[Sequence[int]] = None) -> np.ndarray:
        """``chunk`` tokens per row from ``starts[b]``: write K/V first, then attend
        (decode_step / extend_block, engine/model.py:123-194).  Returns (B, chunk, V)."""
        ids_2d = np.asarray(ids_2d, dtype=np.int64)
        B, chunk = ids_2d.shape
        if slots is None:
            slots = kv.reserve(seq_ids, starts, [chunk] * B)
        h = self._embed(ids_2d.reshape(-1))
        pos = (np.asarray(starts, dtype=np.int64)[:, None] + np.arange(chunk)[None, :]).reshape(-1)

        def fn(i, q, k, v):
            kv.append(i, slots, k, v)
            out = np.zeros(q.shape, dtype=np.float64)
            for b, (sid, st) in enumerate(zip(seq_ids, starts)):
                kk, vv = kv.gather(i, int(sid), int(st) + chunk)
                out[b * chunk:(b + 1) * chunk] = attend(q[b * chunk:(b + 1) * chunk], kk, vv,
                                                        [int(st) + j + 1 for j in range(chunk)])
            return out

        for i in range(self.num_layers):
            h = self._layer(i, h, pos, fn)
        return self._logits(h).reshape(B, chunk, -1)
