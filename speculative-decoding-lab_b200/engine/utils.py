"""Re-export the shared utilities from ``specdec.utils``."""

from __future__ import annotations

from specdec.utils import (  # noqa: F401
    Stopwatch,
    human_bytes,
    mean_std,
    sanitize_for_json,
    save_json,
    set_seed,
    setup_logger,
    sync_device,
    timestamp,
)
