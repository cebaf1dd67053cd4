"""B200-native paged-KV speculative-decoding engine.

Drop-in for the reference's ``engine`` package (sup-zzj/speculative-decoding-lab,
engine/__init__.py): the same public names, backed by the sm_100a kernels of
``lib/libsdl_b200.so`` (paged KV reserve/append/rewind, paged decode/verify
attention, fused rejection sampling, device-side round commit).
"""

from __future__ import annotations

from .attention import (
    full_attention,
    gather_ctx,
    paged_attention,
    paged_attention_decode,
    paged_attention_extend,
    paged_attention_prefill_chunk,
)
from .config import EngineConfig, SamplingConfig, WorkloadConfig, WorkloadRequest, build_workload
from .kv import BlockAllocator, BlockExhaustedError, PagedKVCache
from .model import RMSNorm, ToyConfig, ToyPagedLM, ToyTokenizer, apply_rotary, make_rotary_cache, rotate_half
from .qwen import QwenPagedModel, build_paged_model, build_random_model, shape_config
from .scheduler import PagedScheduler, SchedulerResult, Sequence, build_kv
from .spec_scheduler import SpeculativePagedScheduler, batch_accept

__version__ = "0.1.0-b200"

__all__ = [
    "BlockAllocator",
    "BlockExhaustedError",
    "EngineConfig",
    "PagedKVCache",
    "PagedScheduler",
    "QwenPagedModel",
    "RMSNorm",
    "SchedulerResult",
    "SamplingConfig",
    "Sequence",
    "SpeculativePagedScheduler",
    "ToyConfig",
    "ToyPagedLM",
    "ToyTokenizer",
    "WorkloadConfig",
    "WorkloadRequest",
    "apply_rotary",
    "batch_accept",
    "build_kv",
    "build_paged_model",
    "build_random_model",
    "build_workload",
    "full_attention",
    "gather_ctx",
    "make_rotary_cache",
    "paged_attention",
    "paged_attention_decode",
    "paged_attention_extend",
    "paged_attention_prefill_chunk",
    "rotate_half",
    "shape_config",
]
