"""Per-step events and the run summary (reference ``engine/metrics.py`` and ``engine/results.py``).

``run_scheduler`` returns a ``ScheduleResult`` with the reference's fields and definitions —
``sequences``, ``metrics``, ``memory``, ``trace``, ``batch_size``, ``batch_info``,
``schedule_metrics``, ``events``, ``request_metrics``, ``batching_method``, ``kv_cache_config``,
``padded_output_tokens()`` (reference ``engine/results.py:75-105``, ``engine/metrics.py:21-269,
292-460``) — plus this package's additions: ``ScheduleMetrics.decode_tok_s`` = decode-step tokens
* 1000 / decode-step ms (the engine decode throughput the benchmark reports; mixed steps are in
``throughput_tok_s`` and ``num_mixed_steps``), ``model_ms``, ``decode_tokens``, ``decode_ms``,
``e2e_wall_ms``, ``paged_cache`` and ``extra`` (host/device bytes, graph replays).  Percentiles are
nearest-rank (reference ``utils.py:7-13``).  Where the reference counts PREFILL steps (prompt
throughput, padding efficiency, prefill chunks), mixed steps are not counted: with the reference's
schedules (mixed off) there are none.
"""

from __future__ import annotations

import math
from collections.abc import Sequence
from dataclasses import dataclass, field
from typing import Any

import torch

from mini_infra_b200.core.request import RequestState
from mini_infra_b200.core.scheduler import SchedulePhase
from mini_infra_b200.core.types import (
    BatchingMethod, DenseCacheConfig, KVCacheConfig, RequestMetrics, SequenceOutput,
)

_MIB = 1024**2


def percentile(values: Sequence[float], percent: float) -> float:
    """Nearest-rank percentile: the ceil(n * p / 100)-th smallest value (at least the first); 0 when empty."""
    if not values:
        return 0.0
    ordered = sorted(values)
    rank = min(max(1, math.ceil(len(ordered) * percent / 100)), len(ordered))
    return ordered[rank - 1]


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
    block_size: int = 0
    bytes_per_block: int = 0
    num_blocks: int = 0
    peak_used_blocks: int = 0
    block_cold_allocation_count: int = 0
    block_reuse_count: int = 0
    block_release_count: int = 0

    def to_dict(self) -> dict[str, Any]:
        return dict(self.__dict__)


@dataclass(frozen=True)
class KVCacheProfile:
    peak_live_kv_cache_mb: float = 0.0
    peak_kv_cache_pool_mb: float = 0.0
    cache_realign_moved_bytes: int = 0
    accessed_kv_cache_tokens: int = 0
    paged_cache: PagedCacheProfile | None = None

    def to_dict(self) -> dict[str, Any]:
        out = {k: v for k, v in self.__dict__.items() if k != "paged_cache"}
        if self.paged_cache is not None:
            out["paged_cache"] = self.paged_cache.to_dict()
        return out


@dataclass(frozen=True)
class MemoryProfile:
    baseline_mb: float = 0.0
    prefill_mb: float | None = 0.0
    peak_allocated_mb: float = 0.0
    peak_reserved_mb: float = 0.0
    weights_mb: float | None = None
    kv_cache: KVCacheProfile = field(default_factory=KVCacheProfile)

    @property
    def dynamic_peak_mb(self) -> float:
        return max(0.0, self.peak_allocated_mb - self.baseline_mb)

    @property
    def fragmentation_mb(self) -> float:
        return max(0.0, self.peak_reserved_mb - self.peak_allocated_mb)

    def to_dict(self) -> dict[str, Any]:
        return {"weights_mb": self.weights_mb, "baseline_allocated_mb": self.baseline_mb,
                "prefill_allocated_mb": self.prefill_mb, "peak_allocated_mb": self.peak_allocated_mb,
                "dynamic_peak_mb": self.dynamic_peak_mb, "peak_reserved_mb": self.peak_reserved_mb,
                "fragmentation_mb": self.fragmentation_mb, "kv_cache": self.kv_cache.to_dict()}


@dataclass(frozen=True)
class GenerationTrace:
    step_latencies_ms: list[float]
    num_active_tokens_per_step: list[int]
    logits_trace: list[torch.Tensor] | None = None


@dataclass(frozen=True)
class BatchScheduleInfo:
    padding_efficiency: float
    slot_utilization: float
    running_capacity_utilization: float | None = None


@dataclass(frozen=True)
class StepAggregatedMetrics:
    ttft_ms: float | None = None
    mean_tpot_ms: float | None = None
    p50_tpot_ms: float | None = None
    p95_tpot_ms: float | None = None
    e2e_wall_ms: float = 0.0
    e2e_model_ms: float = 0.0
    throughput_tok_s: float = 0.0
    throughput_req_s: float = 0.0
    gpu_time_ratio: float | None = None
    effective_prompt_tok_s: float | None = None
    padded_prompt_tok_s: float | None = None


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
    # the reference's remaining fields (logical-clock latencies of the requests)
    makespan_ms: float = 0.0
    cache_management_fraction: float = 0.0
    queue_ms_p50: float = 0.0
    queue_ms_p95: float = 0.0
    ttft_ms_p50: float = 0.0
    ttft_ms_p95: float = 0.0
    end_to_end_ms_p50: float = 0.0
    end_to_end_ms_p95: float = 0.0
    itl_ms_p50: float = 0.0
    itl_ms_p95: float = 0.0
    itl_ms_max: float = 0.0
    max_consecutive_prefill_steps: int = 0
    num_oversize_prefill_steps: int = 0
    num_prefill_chunks: int = 0


@dataclass(frozen=True)
class ScheduleResult:
    sequences: list[SequenceOutput]
    request_metrics: list[RequestMetrics]
    events: list[ScheduleEvent]
    schedule_metrics: ScheduleMetrics
    e2e_wall_ms: float
    paged_cache: PagedCacheProfile | None = None
    extra: dict = field(default_factory=dict)
    metrics: StepAggregatedMetrics = field(default_factory=StepAggregatedMetrics)
    memory: MemoryProfile = field(default_factory=MemoryProfile)
    trace: GenerationTrace | None = None
    batch_size: int = 0
    batch_info: BatchScheduleInfo | None = None
    batching_method: BatchingMethod = BatchingMethod.CONTINUOUS
    kv_cache_config: KVCacheConfig = field(default_factory=DenseCacheConfig)

    @property
    def requests(self) -> list[RequestMetrics]:
        """The per-request metrics (``request_metrics``)."""
        return self.request_metrics

    def padded_output_tokens(self, request_idx: int | Sequence[int] | None = None,
                             pad_token_id: int = 0) -> torch.Tensor:
        """One request's tokens as a 1D tensor (int), or the selected requests' (a sequence of ids,
        in that order; None: all) right-padded into [n, longest] (reference ``engine/results.py:33-72``)."""
        by_id = {s.request_idx: s for s in self.sequences}
        if isinstance(request_idx, int):
            if request_idx not in by_id:
                raise IndexError(f"Request index {request_idx} not found in sequences")
            return torch.tensor(by_id[request_idx].token_ids, dtype=torch.long)
        if request_idx is None:
            chosen = list(self.sequences)
        else:
            missing = [i for i in request_idx if i not in by_id]
            if missing:
                raise IndexError(f"Request index {missing[0]} not found in sequences")
            chosen = [by_id[i] for i in request_idx]
        if not chosen:
            return torch.empty((0, 0), dtype=torch.long)
        out = torch.full((len(chosen), max(s.output_len for s in chosen)), pad_token_id, dtype=torch.long)
        for row, s in enumerate(chosen):
            if s.token_ids:
                out[row, : s.output_len] = torch.tensor(s.token_ids, dtype=torch.long)
        return out


def _longest_prefill_run(events: Sequence[ScheduleEvent]) -> int:
    longest = run = 0
    for e in events:
        run = run + 1 if e.phase is SchedulePhase.PREFILL else 0
        longest = max(longest, run)
    return longest


def summarize_schedule(
    states: Sequence[RequestState],
    events: Sequence[ScheduleEvent],
    max_running_requests: int,
    e2e_wall_ms: float,
    paged_cache: PagedCacheProfile | None,
    *,
    batching_method: BatchingMethod = BatchingMethod.CONTINUOUS,
    kv_cache_config: KVCacheConfig | None = None,
    peak_allocated_mb: float = 0.0,
    peak_reserved_mb: float = 0.0,
    baseline_mb: float = 0.0,
    is_cuda: bool = False,
) -> ScheduleResult:
    """The run's result from the final request states and the event list (reference
    ``engine/metrics.py:326-460``; the definitions of every reference field are kept)."""
    finished_at = {i: n + 1 for n, e in enumerate(events) for i in e.finished_request_ids}
    sequences = [s.to_sequence_output(finished_at.get(s.request.request_idx, len(events))) for s in states]
    requests = [s.to_request_metrics() for s in states]
    busy = sum(e.step_ms for e in events)
    model_ms = sum(e.model_ms for e in events)
    cache_ms = sum(e.cache_management_ms for e in events)
    decode = [e for e in events if e.phase is SchedulePhase.DECODE]
    prefill = [e for e in events if e.phase is SchedulePhase.PREFILL]
    prefill_ms = sum(e.step_ms for e in prefill)
    out_tokens = sum(r.num_output_tokens for r in requests)
    dec_tokens = sum(e.num_generated_tokens for e in decode)
    dec_ms = sum(e.step_ms for e in decode)
    itls = [x for r in requests for x in r.inter_token_latencies_ms]
    prompt_tokens = sum(s.request.prompt_len for s in states)
    padded_prompt_tokens = sum(e.num_scheduled_tokens for e in prefill) or prompt_tokens
    executed_rows = sum(e.physical_batch_size for e in events)
    per_s = lambda n, ms: n * 1000.0 / ms if ms else 0.0  # noqa: E731
    schedule_metrics = ScheduleMetrics(
        request_count=len(states),
        max_running_requests=max_running_requests,
        busy_ms=busy,
        model_ms=model_ms,
        cache_management_ms=cache_ms,
        scheduler_ms=sum(e.scheduler_ms for e in events),
        num_prefill_steps=len(prefill),
        num_decode_steps=len(decode),
        num_output_tokens=out_tokens,
        throughput_tok_s=per_s(out_tokens, busy),
        decode_tokens=dec_tokens,
        decode_ms=dec_ms,
        decode_tok_s=per_s(dec_tokens, dec_ms),
        max_prefill_step_tokens=max((e.num_scheduled_tokens for e in prefill), default=0),
        max_prefill_step_ms=max((e.step_ms for e in prefill), default=0.0),
        num_mixed_steps=sum(1 for e in events if e.phase is SchedulePhase.MIXED),
        makespan_ms=(max(r.completion_ms for r in requests) - min(r.arrival_ms for r in requests)) if requests else 0.0,
        cache_management_fraction=cache_ms / busy if busy else 0.0,
        queue_ms_p50=percentile([r.queue_ms for r in requests], 50),
        queue_ms_p95=percentile([r.queue_ms for r in requests], 95),
        ttft_ms_p50=percentile([r.ttft_ms for r in requests], 50),
        ttft_ms_p95=percentile([r.ttft_ms for r in requests], 95),
        end_to_end_ms_p50=percentile([r.end_to_end_ms for r in requests], 50),
        end_to_end_ms_p95=percentile([r.end_to_end_ms for r in requests], 95),
        itl_ms_p50=percentile(itls, 50),
        itl_ms_p95=percentile(itls, 95),
        itl_ms_max=max(itls, default=0.0),
        max_consecutive_prefill_steps=_longest_prefill_run(events),
        num_oversize_prefill_steps=sum(1 for e in events if e.is_oversize_prefill),
        num_prefill_chunks=sum(e.physical_batch_size for e in prefill),
    )
    metrics = StepAggregatedMetrics(
        e2e_wall_ms=e2e_wall_ms,
        e2e_model_ms=model_ms,
        throughput_tok_s=per_s(out_tokens, busy),
        throughput_req_s=per_s(len(states), busy),
        gpu_time_ratio=(min(1.0, model_ms / e2e_wall_ms) if e2e_wall_ms > 0 else 0.0) if is_cuda else None,
        effective_prompt_tok_s=per_s(prompt_tokens, prefill_ms),
        padded_prompt_tok_s=per_s(padded_prompt_tokens, prefill_ms),
    )
    memory = MemoryProfile(
        baseline_mb=baseline_mb,
        prefill_mb=None,
        peak_allocated_mb=peak_allocated_mb,
        peak_reserved_mb=peak_reserved_mb,
        kv_cache=KVCacheProfile(
            peak_live_kv_cache_mb=max((e.live_kv_cache_bytes for e in events), default=0) / _MIB,
            peak_kv_cache_pool_mb=max((e.kv_cache_pool_bytes for e in events), default=0) / _MIB,
            cache_realign_moved_bytes=sum(e.cache_realign_moved_bytes for e in events),
            accessed_kv_cache_tokens=sum(e.accessed_kv_cache_tokens for e in events),
            paged_cache=paged_cache,
        ),
    )
    batch_info = BatchScheduleInfo(
        padding_efficiency=prompt_tokens / padded_prompt_tokens if padded_prompt_tokens else 0.0,
        slot_utilization=out_tokens / executed_rows if executed_rows else 0.0,
        running_capacity_utilization=(sum(e.num_active_requests * e.step_ms for e in events)
                                      / (max_running_requests * busy)) if busy else 0.0,
    )
    trace = GenerationTrace([e.step_ms for e in events], [e.num_generated_tokens for e in events])
    return ScheduleResult(
        sequences=sequences, request_metrics=requests, events=list(events), schedule_metrics=schedule_metrics,
        e2e_wall_ms=e2e_wall_ms, paged_cache=paged_cache, metrics=metrics, memory=memory, trace=trace,
        batch_size=len(states), batch_info=batch_info, batching_method=batching_method,
        kv_cache_config=kv_cache_config if kv_cache_config is not None else DenseCacheConfig(),
    )


__all__ = [
    "BatchScheduleInfo",
    "GenerationTrace",
    "KVCacheProfile",
    "MemoryProfile",
    "PagedCacheProfile",
    "ScheduleEvent",
    "ScheduleMetrics",
    "ScheduleResult",
    "StepAggregatedMetrics",
    "percentile",
    "summarize_schedule",
]
