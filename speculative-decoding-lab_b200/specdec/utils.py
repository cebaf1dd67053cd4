"""Small shared utilities: logging, timing, seeding and JSON output."""

from __future__ import annotations

import json
import logging
import math
import os
import random
import sys
import time
from datetime import datetime
from typing import Any, Dict, List, Optional

import numpy as np

_LOG_FORMAT = "%(asctime)s | %(levelname)-7s | %(name)s | %(message)s"


def setup_logger(name: str = "specdec", level: int = logging.INFO) -> logging.Logger:
    """A stdout logger with a timestamped format (one handler per name)."""
    logger = logging.getLogger(name)
    if not logger.handlers:
        handler = logging.StreamHandler(sys.stdout)
        handler.setFormatter(logging.Formatter(_LOG_FORMAT, datefmt="%H:%M:%S"))
        logger.addHandler(handler)
        logger.propagate = False
    logger.setLevel(level)
    return logger


def set_seed(seed: int = 20260920) -> None:
    """Seed Python, numpy and torch RNGs."""
    random.seed(seed)
    np.random.seed(seed)
    os.environ["PYTHONHASHSEED"] = str(seed)
    import torch

    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


def sanitize_for_json(obj: Any) -> Any:
    """Replace NaN/inf with None and numpy scalars with Python numbers."""
    if isinstance(obj, dict):
        return {str(k): sanitize_for_json(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return [sanitize_for_json(v) for v in obj]
    if isinstance(obj, (np.floating, float)):
        v = float(obj)
        return None if (math.isnan(v) or math.isinf(v)) else v
    if isinstance(obj, np.integer):
        return int(obj)
    return obj


def save_json(payload: Dict[str, Any], path: str) -> str:
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "w", encoding="utf-8") as handle:
        json.dump(sanitize_for_json(payload), handle, ensure_ascii=False, indent=2)
    return os.path.abspath(path)


def timestamp() -> str:
    return datetime.now().strftime("%Y%m%d_%H%M%S")


class Stopwatch:
    """Context manager measuring wall-clock latency in milliseconds."""

    def __init__(self) -> None:
        self.elapsed_ms: float = 0.0
        self._start: float = 0.0

    def __enter__(self) -> "Stopwatch":
        self._start = time.perf_counter()
        return self

    def __exit__(self, *exc_info: Any) -> None:
        self.elapsed_ms = (time.perf_counter() - self._start) * 1000.0


def sync_device(device: Any) -> None:
    """Synchronise CUDA so wall-clock timings are meaningful."""
    import torch

    if str(device).startswith("cuda") and torch.cuda.is_available():
        torch.cuda.synchronize()


def human_bytes(num_bytes: float) -> str:
    for unit in ("B", "KB", "MB", "GB"):
        if abs(num_bytes) < 1024.0:
            return "{:.1f}{}".format(num_bytes, unit)
        num_bytes /= 1024.0
    return "{:.1f}TB".format(num_bytes)


def mean_std(values: List[float]) -> Dict[str, Optional[float]]:
    """Mean / sample std of a list, tolerating empty input."""
    if not values:
        return {"mean": None, "std": None, "n": 0}
    array = np.asarray(values, dtype=np.float64)
    return {
        "mean": float(array.mean()),
        "std": float(array.std(ddof=1)) if array.size > 1 else 0.0,
        "n": int(array.size),
    }
