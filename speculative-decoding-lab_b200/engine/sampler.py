"""Seeded generation helpers for the serving engine (engine/sampler.py:20-24)."""

from __future__ import annotations

from typing import Optional

import torch

from specdec.sampler import UniformStream  # noqa: F401
from specdec.sampler import build_generator as _build_generator

__all__ = ["build_generator", "UniformStream"]


def build_generator(seed: int, device: Optional[torch.device] = None) -> torch.Generator:
    """Deterministic CPU generator seeded with ``seed``."""
    return _build_generator(seed, device)
