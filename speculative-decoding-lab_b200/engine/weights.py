"""Deterministic numpy weights for parity runs of the Qwen-shaped models.

``qwen_numpy_state(config, seed, std)`` draws every projection / embedding
weight and bias from ``numpy.random.default_rng(seed)`` as N(0, std) float32
in one fixed name order, with RMSNorm weights = 1.  The same arrays can be
loaded into this engine's ``QwenPagedModel`` and into the reference's, so both
run bit-identical weights (the golden-fixture generator relies on it).
"""

from __future__ import annotations

from typing import Any, Dict, List, Tuple

import numpy as np


def qwen_param_shapes(config: Any) -> List[Tuple[str, Tuple[int, ...]]]:
    """``transformers``-style parameter names and shapes, in draw order."""
    H = int(config.hidden_size)
    nq = int(config.num_attention_heads)
    nkv = int(getattr(config, "num_key_value_heads", nq))
    d = int(getattr(config, "head_dim", 0) or H // nq)
    F = int(config.intermediate_size)
    V = int(config.vocab_size)
    bias = bool(getattr(config, "attention_bias", True))
    out: List[Tuple[str, Tuple[int, ...]]] = [("embed_tokens.weight", (V, H))]
    for i in range(int(config.num_hidden_layers)):
        p = "layers.{}.".format(i)
        out.append((p + "input_layernorm.weight", (H,)))
        out.append((p + "self_attn.q_proj.weight", (nq * d, H)))
        if bias:
            out.append((p + "self_attn.q_proj.bias", (nq * d,)))
        out.append((p + "self_attn.k_proj.weight", (nkv * d, H)))
        if bias:
            out.append((p + "self_attn.k_proj.bias", (nkv * d,)))
        out.append((p + "self_attn.v_proj.weight", (nkv * d, H)))
        if bias:
            out.append((p + "self_attn.v_proj.bias", (nkv * d,)))
        out.append((p + "self_attn.o_proj.weight", (H, nq * d)))
        out.append((p + "post_attention_layernorm.weight", (H,)))
        out.append((p + "mlp.gate_proj.weight", (F, H)))
        out.append((p + "mlp.up_proj.weight", (F, H)))
        out.append((p + "mlp.down_proj.weight", (H, F)))
    out.append(("norm.weight", (H,)))
    if not bool(getattr(config, "tie_word_embeddings", False)):
        out.append(("lm_head.weight", (V, H)))
    return out


def qwen_numpy_state(config: Any, seed: int, std: float = 0.02) -> Dict[str, np.ndarray]:
    rng = np.random.default_rng(int(seed))
    state: Dict[str, np.ndarray] = {}
    for name, shape in qwen_param_shapes(config):
        if name.endswith("layernorm.weight") or name == "norm.weight":
            state[name] = np.ones(shape, dtype=np.float32)
        else:
            state[name] = (rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)
    return state
