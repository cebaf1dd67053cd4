"""B200-native paged-KV speculative-decoding engine.

Drop-in for the reference's ``engine`` package (sup-zzj/speculative-decoding-lab,
engine/__init__.py): the same public names, backed by the sm_100a kernels of
``lib/libsdl_b200.so`` (paged KV reserve/append/rewind, paged decode/verify
attention, fused rejection sampling, device-side round commit).
"""

from __future__ import annotations

import importlib

# Public names resolve lazily (PEP 562), so ``from engine import _lib`` -- which
# specdec.sampler does -- never re-enters modules that import specdec.sampler.
_EXPORTS = {
    "full_attention": ".attention",
    "gather_ctx": ".attention",
    "paged_attention": ".attention",
    "paged_attention_decode": ".attention",
    "paged_attention_extend": ".attention",
    "paged_attention_prefill_chunk": ".attention",
    "EngineConfig": ".config",
    "SamplingConfig": ".config",
    "WorkloadConfig": ".config",
    "WorkloadRequest": ".config",
    "build_workload": ".config",
    "BlockAllocator": ".kv",
    "BlockExhaustedError": ".kv",
    "PagedKVCache": ".kv",
    "RMSNorm": ".model",
    "ToyConfig": ".model",
    "ToyPagedLM": ".model",
    "ToyTokenizer": ".model",
    "apply_rotary": ".model",
    "make_rotary_cache": ".model",
    "rotate_half": ".model",
    "QwenPagedModel": ".qwen",
    "build_paged_model": ".qwen",
    "build_random_model": ".qwen",
    "shape_config": ".qwen",
    "PagedScheduler": ".scheduler",
    "SchedulerResult": ".scheduler",
    "Sequence": ".scheduler",
    "build_kv": ".scheduler",
    "SpeculativePagedScheduler": ".spec_scheduler",
    "batch_accept": ".spec_scheduler",
}


def __getattr__(name):
    mod = _EXPORTS.get(name)
    if mod is None:
        raise AttributeError("module 'engine' has no attribute {!r}".format(name))
    value = getattr(importlib.import_module(mod, __name__), name)
    globals()[name] = value
    return value


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
