"""Qwen2-style paged model (engine/qwen.py:34-431) on the B200 kernels.

Parameter names mirror ``transformers`` (``layers.N.self_attn.q_proj`` ...), so
a state dict transfers in one call; q/k/v projections carry biases
(``attention_bias``, engine/qwen.py:50-55).  The forward path is the shared
``PagedLMMixin`` one (batched reserve + one append and one paged-attention
launch per layer).  The reference runs a discarded attention before the K/V
write in ``decode_step`` (engine/qwen.py:120); it has no effect on results and
is not reproduced.

No checkpoints are reachable here, so :func:`build_random_model` makes
random-init models of the benchmark shapes; :func:`build_paged_model` loads a
local ``transformers`` checkpoint when one exists.
"""

from __future__ import annotations

import os
from typing import Any, Dict, List, Optional, Sequence

import torch
from torch import nn

from . import layer_ops
from .model import IdTokenizer, PagedLMMixin, RMSNorm, apply_rotary, apply_rotary_, make_rotary_cache, paged_attend
from .utils import setup_logger

logger = setup_logger(__name__)


class QwenAttention(nn.Module):
    def __init__(self, hidden: int, num_q_heads: int, num_kv_heads: int, head_dim: int,
                 attention_bias: bool = True) -> None:
        super().__init__()
        self.num_heads = num_q_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.q_proj = nn.Linear(hidden, num_q_heads * head_dim, bias=attention_bias)
        self.k_proj = nn.Linear(hidden, num_kv_heads * head_dim, bias=attention_bias)
        self.v_proj = nn.Linear(hidden, num_kv_heads * head_dim, bias=attention_bias)
        self.o_proj = nn.Linear(num_q_heads * head_dim, hidden, bias=False)

    def qkv_fused(self, x: torch.Tensor) -> torch.Tensor:
        """q, k and v projections as one GEMM over the concatenated weights:
        rows of ``[q heads | k heads | v heads] x head_dim``.  The
        concatenation is cached and rebuilt when a projection's storage or
        in-place version changes."""
        parts = [self.q_proj, self.k_proj, self.v_proj]
        params = [m.weight for m in parts] + [m.bias for m in parts if m.bias is not None]
        key = tuple((t.data_ptr(), t._version, t.dtype) for t in params)
        if self.__dict__.get("_qkv_key") != key:
            w = torch.cat([m.weight for m in parts], 0)
            b = torch.cat([m.bias for m in parts], 0) if all(m.bias is not None for m in parts) else None
            self.__dict__["_qkv"] = (w, b)
            self.__dict__["_qkv_key"] = key
        w, b = self.__dict__["_qkv"]
        return torch.nn.functional.linear(x, w, b)


class QwenMLP(nn.Module):
    def __init__(self, hidden: int, intermediate: int) -> None:
        super().__init__()
        self.gate_proj = nn.Linear(hidden, intermediate, bias=False)
        self.up_proj = nn.Linear(hidden, intermediate, bias=False)
        self.down_proj = nn.Linear(intermediate, hidden, bias=False)

    def gate_up_fused(self, x: torch.Tensor) -> torch.Tensor:
        """gate and up projections as one GEMM over the concatenated weights
        (rows ``[gate | up]``); the concatenation is cached and rebuilt when a
        projection's storage or in-place version changes."""
        key = tuple((t.data_ptr(), t._version, t.dtype) for t in (self.gate_proj.weight, self.up_proj.weight))
        if self.__dict__.get("_gu_key") != key:
            self.__dict__["_gu"] = torch.cat([self.gate_proj.weight, self.up_proj.weight], 0)
            self.__dict__["_gu_key"] = key
        return torch.nn.functional.linear(x, self.__dict__["_gu"])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if layer_ops.fusable(x):  # 16-bit models: one gate/up GEMM, one gate launch
            return self.down_proj(layer_ops.swiglu(self.gate_up_fused(x), self.gate_proj.out_features))
        return self.down_proj(torch.nn.functional.silu(self.gate_proj(x)) * self.up_proj(x))


class QwenDecoderLayer(nn.Module):
    """A Qwen2 decoder layer whose names match ``transformers``."""

    def __init__(self, hidden: int, num_q_heads: int, num_kv_heads: int, head_dim: int, intermediate: int,
                 eps: float, attention_bias: bool = True) -> None:
        super().__init__()
        self.input_layernorm = RMSNorm(hidden, eps)
        self.self_attn = QwenAttention(hidden, num_q_heads, num_kv_heads, head_dim, attention_bias)
        self.post_attention_layernorm = RMSNorm(hidden, eps)
        self.mlp = QwenMLP(hidden, intermediate)

    def forward_plan(self, hidden, kv, layer_index, plan, cos, sin):
        """One decoder layer.  16-bit models return the residual stream as a
        pair ``(hidden, mlp_out)`` whose sum the next layer's input norm forms
        in its own launch (the same bf16 rounding as ``hidden + mlp_out``);
        ``hidden`` may arrive as such a pair."""
        attn = self.self_attn
        if isinstance(hidden, tuple):
            norm = self.input_layernorm
            hidden, x = layer_ops.add_rmsnorm(hidden[0], hidden[1], norm.weight, norm.eps)
        else:
            x = self.input_layernorm(hidden)
        lead = tuple(hidden.shape[:-1])
        d, hq, hkv = attn.head_dim, attn.num_heads, attn.num_kv_heads
        rope = None
        if layer_ops.fusable(x):
            # 16-bit models: one projection GEMM; RoPE rides the attention
            # launch (q rotated as it is loaded, k as it is stored), or -- when
            # the rows are stored before attending -- one launch over the q
            # and k heads, which sit side by side in each row of its output
            qkv = attn.qkv_fused(x)
            qk = qkv[..., :(hq + hkv) * d].view(*lead, hq + hkv, d)
            if plan.append_first:
                layer_ops.rope_(qk, sin, cos)
            else:
                rope = (cos, sin)
            q, k = qk[..., :hq, :], qk[..., hq:, :]
            v = qkv[..., (hq + hkv) * d:].view(*lead, hkv, d)
        else:
            q = apply_rotary_(attn.q_proj(x).view(*lead, hq, d), sin, cos)
            k = apply_rotary_(attn.k_proj(x).view(*lead, hkv, d), sin, cos)
            v = attn.v_proj(x).view(*lead, hkv, d)
        out = paged_attend(q, k, v, kv, layer_index, plan, rope=rope)
        o = attn.o_proj(out.reshape(*lead, -1))
        if layer_ops.fusable(hidden):  # residual add + post-attention norm in one launch
            norm = self.post_attention_layernorm
            hidden, x2 = layer_ops.add_rmsnorm(hidden, o, norm.weight, norm.eps)
            return hidden, self.mlp(x2)
        hidden = hidden + o
        return hidden + self.mlp(self.post_attention_layernorm(hidden))


class QwenPagedModel(PagedLMMixin, nn.Module):
    """A Qwen2.5-shaped causal LM whose forward consumes ``PagedKVCache``."""

    def __init__(self, config: Any, device: torch.device) -> None:
        super().__init__()
        self.config = config
        self.device = torch.device(device)
        self.num_layers = int(config.num_hidden_layers)
        self.num_q_heads = int(config.num_attention_heads)
        self.num_kv_heads = int(getattr(config, "num_key_value_heads", self.num_q_heads))
        self._head_dim = int(getattr(config, "head_dim", 0) or (config.hidden_size // self.num_q_heads))
        self._theta = float(getattr(config, "rope_theta", 10000.0))
        self._eps = float(getattr(config, "rms_norm_eps", 1e-6))
        self._max_len = int(getattr(config, "max_position_embeddings", 2048))
        self._attn_bias = bool(getattr(config, "attention_bias", True))
        self.vocab_size = int(config.vocab_size)
        self._tie = bool(getattr(config, "tie_word_embeddings", False))
        self.embed_tokens = nn.Embedding(self.vocab_size, int(config.hidden_size))
        self.layers = nn.ModuleList(
            [
                QwenDecoderLayer(int(config.hidden_size), self.num_q_heads, self.num_kv_heads, self._head_dim,
                                 int(config.intermediate_size), self._eps, self._attn_bias)
                for _ in range(self.num_layers)
            ]
        )
        self.norm = RMSNorm(int(config.hidden_size), self._eps)
        self.lm_head = nn.Linear(int(config.hidden_size), self.vocab_size, bias=False)
        if self._tie:
            self.lm_head.weight = self.embed_tokens.weight
        # One RoPE table (the reference keeps an identical copy per layer and
        # reads layer 0's, engine/qwen.py:59-61,272-274); cast with the model.
        self.register_buffer("_cos_sin", make_rotary_cache(self._head_dim, self._theta, self._max_len,
                                                           torch.device("cpu")), persistent=False)
        self.forward_calls = 0
        self.tokenizer = IdTokenizer(self.vocab_size, getattr(config, "eos_token_id", None))

    @property
    def head_dim(self) -> int:
        return self._head_dim

    @property
    def dtype(self) -> torch.dtype:
        return next(self.parameters()).dtype

    def _rope_table(self) -> torch.Tensor:
        return self._cos_sin

    def _logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.lm_head(self.norm(hidden))

    def encode(self, text) -> List[int]:
        return list(self.tokenizer.encode(text))

    def decode_text(self, token_ids: Sequence[int], skip_special_tokens: bool = True) -> str:
        return self.tokenizer.decode(list(token_ids), skip_special_tokens=skip_special_tokens)

    def reset_counters(self) -> None:
        self.forward_calls = 0


# ------------------------------------------------------------- model shapes
from .workloads import QWEN_SHAPES, shape_config  # noqa: E402,F401


def build_random_model(config: Any, device: torch.device, dtype: torch.dtype, seed: int = 0, std: float = 0.02,
                       state_dict: Optional[Dict[str, torch.Tensor]] = None) -> QwenPagedModel:
    """Random-init model: every weight and bias ~ N(0, std), norms = 1.

    With ``state_dict`` the given weights are loaded instead (e.g. the numpy
    weights of :func:`engine.weights.qwen_numpy_state`).
    """
    device = torch.device(device)
    with torch.device(device):
        model = QwenPagedModel(config, device)
    model.to(dtype=dtype)
    model._cos_sin = model._cos_sin.to(device=device, dtype=dtype)
    if state_dict is not None:
        missing, unexpected = model.load_state_dict(state_dict, strict=False)
        if missing:
            raise RuntimeError("missing weights: {}".format(missing))
    else:
        gen = torch.Generator(device=device)
        gen.manual_seed(int(seed))
        with torch.no_grad():
            for name, p in model.named_parameters():
                if name.endswith("layernorm.weight") or name == "norm.weight":
                    p.fill_(1.0)
                else:
                    p.copy_(torch.randn(p.shape, generator=gen, device=device, dtype=torch.float32).mul_(std))
    model.requires_grad_(False)
    model.eval()
    return model


def build_paged_model(model_id: str, cache_dir: str, device: torch.device, dtype: torch.dtype) -> QwenPagedModel:
    """Load local ``transformers`` Qwen2 weights into the paged engine."""
    from transformers import AutoConfig, AutoModelForCausalLM, AutoTokenizer

    source = model_id
    for cand in (model_id, os.path.join(cache_dir, model_id), os.path.join(cache_dir, os.path.basename(model_id))):
        if os.path.isdir(cand):
            source = cand
            break
    config = AutoConfig.from_pretrained(source, cache_dir=cache_dir)
    native = AutoModelForCausalLM.from_pretrained(source, cache_dir=cache_dir, torch_dtype=dtype)
    state = {(k[6:] if k.startswith("model.") else k): v for k, v in native.state_dict().items()}
    model = build_random_model(config, device, dtype, state_dict=state)
    model.tokenizer = AutoTokenizer.from_pretrained(source, cache_dir=cache_dir)
    del native
    return model


def load_pair(draft_id: str, target_id: str, cache_dir: str, device: torch.device, dtype: torch.dtype):
    """Returns ``(draft_model, target_model)`` (engine/qwen.py:413-431)."""
    target = build_paged_model(target_id, cache_dir, device, dtype)
    draft = build_paged_model(draft_id, cache_dir, device, dtype)
    return draft, target
