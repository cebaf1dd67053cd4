"""Host-side helpers the engine needs: a named logger, a wall-clock timer that
includes the device, and a summary of a list of latencies."""

from __future__ import annotations

import logging
import statistics
import sys
import time
from typing import Any, Dict, List, Optional


def setup_logger(name: str = "specdec", level: int = logging.INFO) -> logging.Logger:
    """Logger ``name`` writing ``HH:MM:SS LEVEL name: message`` lines to stdout.

    Calling it again for the same name reuses the handler already attached.
    """
    log = logging.getLogger(name)
    if not any(getattr(h, "_sdl_handler", False) for h in log.handlers):
        h = logging.StreamHandler(sys.stdout)
        h.setFormatter(logging.Formatter("%(asctime)s %(levelname)s %(name)s: %(message)s", "%H:%M:%S"))
        h._sdl_handler = True  # type: ignore[attr-defined]
        log.addHandler(h)
        log.propagate = False
    log.setLevel(level)
    return log


def sync_device(device: Any) -> None:
    """Wait for the CUDA device behind ``device`` (no-op for a CPU device)."""
    import torch

    dev = torch.device(device)
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)


class Stopwatch:
    """``with Stopwatch() as w: ...`` leaves the block's duration in
    ``w.elapsed_ms`` (host clock; synchronise the device inside the block to
    include queued GPU work)."""

    def __init__(self) -> None:
        self.elapsed_ms = 0.0
        self._t0 = 0.0

    def __enter__(self) -> "Stopwatch":
        self._t0 = time.perf_counter()
        return self

    def __exit__(self, *_exc: Any) -> None:
        self.elapsed_ms = 1e3 * (time.perf_counter() - self._t0)


def mean_std(values: List[float]) -> Dict[str, Optional[float]]:
    """``{"mean", "std", "n"}`` of ``values``: ``std`` is the sample standard
    deviation (0.0 for a single value); an empty list gives ``None`` for both."""
    n = len(values)
    if n == 0:
        return {"mean": None, "std": None, "n": 0}
    xs = [float(v) for v in values]
    return {"mean": statistics.fmean(xs), "std": statistics.stdev(xs) if n > 1 else 0.0, "n": n}
