"""Backend step contract (reference ``engine/schedule_backend.py``)."""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class ScheduleStepOutput:
    next_tokens: list[int]
    model_ms: float
    cache_ms: float
    physical_batch_size: int
    live_kv_cache_bytes: int
    kv_cache_pool_bytes: int = 0
    cache_realign_moved_bytes: int = 0
    accessed_kv_cache_tokens: int = 0
