"""Engine: configuration, paged backend and the scheduling loop."""

from mini_infra_b200.core.types import BatchingMethod
from mini_infra_b200.engine.config import EngineConfig, validate_engine_config
from mini_infra_b200.engine.metrics import (
    BatchScheduleInfo, GenerationTrace, KVCacheProfile, MemoryProfile, PagedCacheProfile, ScheduleEvent, ScheduleMetrics,
    ScheduleResult, StepAggregatedMetrics,
)
from mini_infra_b200.engine.paged_schedule_backend import PagedScheduleBackend
from mini_infra_b200.engine.schedule_backend import ScheduleStepOutput
from mini_infra_b200.engine.scheduler_loop import run_scheduler

__all__ = [
    "BatchScheduleInfo",
    "BatchingMethod",
    "EngineConfig",
    "GenerationTrace",
    "KVCacheProfile",
    "MemoryProfile",
    "PagedCacheProfile",
    "PagedScheduleBackend",
    "ScheduleEvent",
    "ScheduleMetrics",
    "ScheduleResult",
    "ScheduleStepOutput",
    "StepAggregatedMetrics",
    "run_scheduler",
    "validate_engine_config",
]
