"""Typed configuration shared by the sampler and the schedulers."""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any, Dict


@dataclass
class SamplingConfig:
    """Post-processing applied to raw logits before drawing a token.

    ``temperature <= 0`` selects greedy decoding (a one-hot distribution on the
    argmax token), as in specdec/config.py:19-48 of the reference.
    """

    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0

    @property
    def is_greedy(self) -> bool:
        return self.temperature <= 0.0

    def describe(self) -> str:
        if self.is_greedy:
            return "greedy"
        parts = ["T={:.2f}".format(self.temperature)]
        if self.top_k > 0:
            parts.append("top_k={}".format(self.top_k))
        if self.top_p < 1.0:
            parts.append("top_p={:.2f}".format(self.top_p))
        return ", ".join(parts)

    def to_dict(self) -> Dict[str, Any]:
        payload = asdict(self)
        payload["mode"] = "greedy" if self.is_greedy else "sampling"
        return payload


def validate_gamma(gamma: int) -> int:
    """Guard against meaningless draft lengths (1..32, specdec/config.py:109-115)."""
    if gamma < 1:
        raise ValueError("gamma must be >= 1, got {}".format(gamma))
    if gamma > 32:
        raise ValueError("gamma > 32 is not supported by this implementation")
    return gamma
