"""Typed configuration for the paged engine (engine/config.py:21-147).

Same dataclasses and ``build_workload`` draw order as the reference, so a
seeded workload is identical request for request.  ``WorkloadRequest.prompt``
may also be a sequence of token ids (random-init models have no tokenizer).
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any, Dict, List, Optional, Sequence, Tuple, Union

import torch


@dataclass
class EngineConfig:
    """Model + paged KV parameters for a single serving engine."""

    model_id: str = "Qwen/Qwen2.5-1.5B"
    device: str = "auto"
    dtype: str = "auto"
    cache_dir: str = "models"
    block_size: int = 16
    max_num_blocks: int = 256
    max_batch: int = 16

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)


@dataclass
class SamplingConfig:
    """Decoding temperature; ``temperature <= 0`` selects greedy decoding."""

    temperature: float = 0.0

    @property
    def is_greedy(self) -> bool:
        return self.temperature <= 0.0

    def describe(self) -> str:
        if self.is_greedy:
            return "greedy"
        return "temperature={}".format(self.temperature)

    def to_dict(self) -> Dict[str, Any]:
        return {"temperature": self.temperature, "mode": "greedy" if self.is_greedy else "sampling"}


@dataclass
class WorkloadRequest:
    """One generation request; ``arrive_time`` is in scheduler steps."""

    prompt: Union[str, Sequence[int]]
    max_new_tokens: int
    arrive_time: int = 0

    def to_dict(self) -> Dict[str, Any]:
        d = asdict(self)
        if not isinstance(self.prompt, str):
            d["prompt"] = list(self.prompt)
        return d


@dataclass
class WorkloadConfig:
    """How to synthesise a batch of diverse requests for a serving experiment."""

    prompts: Sequence[str]
    num_requests: int = 8
    min_tokens: int = 8
    max_tokens: int = 32
    arrival_window: int = 4
    seed: int = 20260920

    def to_dict(self) -> Dict[str, Any]:
        payload = asdict(self)
        payload["prompts"] = list(self.prompts)
        return payload


DEFAULT_PROMPTS: Tuple[str, ...] = (
    "The key idea behind a paged attention server is",
    "In a large-scale inference system, continuous batching",
    "The GPU is most underutilised during the decode phase",
    "A KV cache must be re-layouted to fit dynamic request",
    "Scheduling matters more than raw FLOPs for serving",
    "When one request finishes early its slot should be reused",
)


def config_from_namespace(args: Any, base: Optional[EngineConfig] = None) -> EngineConfig:
    config = base or EngineConfig()
    for name in ("model_id", "device", "dtype", "cache_dir", "block_size", "max_num_blocks", "max_batch"):
        src = "model" if name == "model_id" else name
        setattr(config, name, getattr(args, src, getattr(config, name)))
    return config


def build_workload(cfg: WorkloadConfig, generator: Any) -> List[WorkloadRequest]:
    """Sample a heterogeneous request set (budget then arrival per request)."""
    requests: List[WorkloadRequest] = []
    for index in range(cfg.num_requests):
        prompt = cfg.prompts[index % len(cfg.prompts)]
        budget = int(torch.randint(cfg.min_tokens, cfg.max_tokens + 1, (1,), generator=generator).item())
        arrive = int(torch.randint(0, cfg.arrival_window + 1, (1,), generator=generator).item())
        requests.append(WorkloadRequest(prompt=prompt, max_new_tokens=budget, arrive_time=arrive))
    return requests
