"""Per-step events and the run summary (subset of the reference's ``engine/metrics.py``).

``throughput_tok_s`` = generated tokens * 1000 / busy ms, as the reference defines it;
``decode_tok_s`` = decode-step tokens * 1000 / decode-step ms (the engine decode throughput the
benchmark reports; mixed steps are in ``throughput_tok_s`` and ``num_mixed_steps``, not here).
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass, field

from mini_infra_b200.core.request import RequestState
from mini_infra_b200.core.scheduler import SchedulePhase
from mini_infra_b200.core.types import RequestMetrics, SequenceOutput


@dataclass(frozen=True)
class ScheduleEvent:
    phase: SchedulePhase
    admitted_request_ids: tuple[int, ...]
    finished_request_ids: tuple[int, ...]
    physical_batch_size: int
    num_active_requests: int
    num_generated_tokens: int
    num_scheduled_tokens: int
    step_ms: float
    model_ms: float
    cache_management_ms: float
    scheduler_ms: float
    live_kv_cache_bytes: int
    kv_cache_pool_bytes: int = 0
    cache_realign_moved_bytes: int = 0
    accessed_kv_cache_tokens: int = 0
    is_oversize_prefill: bool = False


@dataclass(frozen=True)
class PagedCacheProfile:
    block_size: int
    bytes_per_block: int
    num_blocks: int
    peak_used_blocks: int
    block_cold_allocation_count: int
    block_reuse_count: int
    block_release_count: int


@dataclass(frozen=True)
class ScheduleMetrics:
    request_count: int
    max_running_requests: int
    busy_ms: float
    model_ms: float
    cache_management_ms: float
    scheduler_ms: float
    num_prefill_steps: int
    num_decode_steps: int
    num_output_tokens: int
    throughput_tok_s: float
    decode_tokens: int
    decode_ms: float
    decode_tok_s: float
    max_prefill_step_tokens: int
    max_prefill_step_ms: float
    num_mixed_steps: int = 0  # ChunkedPrefillConfig(mixed=True): steps holding decode rows and chunks


@dataclass(frozen=True)
class ScheduleResult:
    sequences: list[SequenceOutput]
    requests: list[RequestMetrics]
    events: list[ScheduleEvent]
    schedule_metrics: ScheduleMetrics
    e2e_wall_ms: float
    paged_cache: PagedCacheProfile | None = None
    extra: dict = field(default_factory=dict)


def summarize_schedule(
    states: Sequence[RequestState],
    events: Sequence[ScheduleEvent],
    max_running_requests: int,
    e2e_wall_ms: float,
    paged_cache: PagedCacheProfile | None,
) -> ScheduleResult:
    finished_at = {i: n + 1 for n, e in enumerate(events) for i in e.finished_request_ids}
    sequences = [s.to_sequence_output(finished_at.get(s.request.request_idx, len(events))) for s in states]
    requests = [s.to_request_metrics() for s in states]
    busy = sum(e.step_ms for e in events)
    decode = [e for e in events if e.phase is SchedulePhase.DECODE]
    prefill = [e for e in events if e.phase is SchedulePhase.PREFILL]
    out_tokens = sum(r.num_output_tokens for r in requests)
    dec_tokens = sum(e.num_generated_tokens for e in decode)
    dec_ms = sum(e.step_ms for e in decode)
    metrics = ScheduleMetrics(
        request_count=len(states),
        max_running_requests=max_running_requests,
        busy_ms=busy,
        model_ms=sum(e.model_ms for e in events),
        cache_management_ms=sum(e.cache_management_ms for e in events),
        scheduler_ms=sum(e.scheduler_ms for e in events),
        num_prefill_steps=len(prefill),
        num_decode_steps=len(decode),
        num_output_tokens=out_tokens,
        throughput_tok_s=out_tokens * 1000.0 / busy if busy else 0.0,
        decode_tokens=dec_tokens,
        decode_ms=dec_ms,
        decode_tok_s=dec_tokens * 1000.0 / dec_ms if dec_ms else 0.0,
        max_prefill_step_tokens=max((e.num_scheduled_tokens for e in prefill), default=0),
        max_prefill_step_ms=max((e.step_ms for e in prefill), default=0.0),
        num_mixed_steps=sum(1 for e in events if e.phase is SchedulePhase.MIXED),
    )
    return ScheduleResult(sequences, requests, list(events), metrics, e2e_wall_ms, paged_cache)
