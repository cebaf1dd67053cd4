"""The engine's helpers are the ones in ``specdec.utils`` (same module path as
the reference's ``engine/utils.py`` import sites)."""

from __future__ import annotations

from specdec.utils import Stopwatch, mean_std, setup_logger, sync_device  # noqa: F401
