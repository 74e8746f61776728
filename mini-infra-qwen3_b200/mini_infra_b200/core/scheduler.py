"""Iteration-level scheduler (no torch): arrival / waiting / running queues and per-step decisions.

Same behaviour as the reference's ``core/scheduler.py``, which decides every shape the paged
kernels see:

* admission takes the FCFS prefix of the waiting queue allowed by the batching method
  (continuous: any free batch slot; fixed: only when nothing runs), by free batch slots and, for
  the paged cache, by free blocks after reserving what in-flight chunked prefills still need;
* ``prefill-first`` prefills all admissible prompts whole, else decodes;
* ``token-budget`` caps a whole-prompt prefill at ``token_budget`` padded tokens (a lone
  over-budget head request runs alone) and never runs two prefills back to back while requests
  are running (decode protection);
* ``chunked-prefill`` gives every candidate (in-flight prefills first, then admissible new
  requests) a chunk of at most ``token_budget // n_candidates`` prompt tokens, with the same
  decode protection; prefill and decode steps stay phase-exclusive;
* ``chunked-prefill`` with ``mixed=True`` (not in the reference): a step holds every decoding
  request (one token each) and the chunks planned from ``token_budget - n_decoding`` tokens
  (at most that many candidates, so every chunk has a token); with both present it is a
  ``MIXED`` step, otherwise a plain prefill or decode step.
"""

from __future__ import annotations

import heapq
from collections import deque
from collections.abc import Iterable, Sequence
from dataclasses import dataclass
from enum import Enum

from mini_infra_b200.core.block_manager import KVCacheManager, num_blocks_for_tokens
from mini_infra_b200.core.request import Request, RequestState, RequestStatus, validate_requests
from mini_infra_b200.core.types import BatchingMethod, ChunkedPrefillConfig, PrefillFirstConfig, SchedulerConfig


class ArrivalQueue:
    """Future requests ordered by arrival time (stable, so ties keep submission order)."""

    def __init__(self, states: Iterable[RequestState]):
        self._q: deque[RequestState] = deque(sorted(states, key=lambda s: s.request.arrival_ms))

    def __len__(self) -> int:
        return len(self._q)

    def __bool__(self) -> bool:
        return bool(self._q)

    def __iter__(self):
        return iter(self._q)

    def pop_arrived(self, clock_ms: float) -> list[RequestState]:
        out = []
        while self._q and self._q[0].request.arrival_ms <= clock_ms:
            out.append(self._q.popleft())
        return out

    def next_arrival_ms(self) -> float:
        return self._q[0].request.arrival_ms


class WaitingQueue:
    """Arrived requests without a batch slot, FCFS."""

    def __init__(self, states: Iterable[RequestState] | None = None):
        self._q: deque[RequestState] = deque()
        if states:
            self.extend(states)

    def __len__(self) -> int:
        return len(self._q)

    def __bool__(self) -> bool:
        return bool(self._q)

    def __iter__(self):
        return iter(self._q)

    @property
    def requests(self) -> tuple[RequestState, ...]:
        return tuple(self._q)

    def append(self, state: RequestState) -> None:
        state.status = RequestStatus.WAITING
        self._q.append(state)

    def extend(self, states: Iterable[RequestState]) -> None:
        for s in states:
            self.append(s)

    def pop_batch(self, limit: int) -> list[RequestState]:
        out = []
        while self._q and len(out) < limit:
            out.append(self._q.popleft())
        return out


class RunningQueue:
    """Requests holding a batch slot (including chunked prefills not yet complete)."""

    def __init__(self, capacity: int):
        if capacity < 1:
            raise ValueError(f"capacity must be positive (必须大于 0), got {capacity}")
        self.capacity = capacity
        self._running: list[RequestState] = []
        self._free_slots = list(range(capacity))
        heapq.heapify(self._free_slots)

    def __len__(self) -> int:
        return len(self._running)

    def __bool__(self) -> bool:
        return bool(self._running)

    def __iter__(self):
        return iter(self._running)

    @property
    def free_batch_slots(self) -> tuple[int, ...]:
        return tuple(self._free_slots)

    @property
    def num_free_batch_slots(self) -> int:
        return len(self._free_slots)

    @property
    def requests(self) -> tuple[RequestState, ...]:
        return tuple(self._running)

    @property
    def prefilling_requests(self) -> tuple[RequestState, ...]:
        return tuple(s for s in self._running if s.is_prefilling)

    @property
    def decoding_requests(self) -> tuple[RequestState, ...]:
        return tuple(s for s in self._running if not s.is_prefilling)

    def can_admit(self) -> bool:
        return bool(self._free_slots)

    def admit(self, states: Sequence[RequestState], clock_ms: float) -> list[RequestState]:
        if len(states) > len(self._free_slots):
            raise ValueError(f"not enough batch slots (可用 batch slot 不足): need {len(states)}, have {len(self._free_slots)}")
        for s in states:
            s.status = RequestStatus.RUNNING
            s.admitted_ms = clock_ms
            s.batch_slot_idx = heapq.heappop(self._free_slots)
            self._running.append(s)
        return list(states)

    def process_step_output(
        self,
        token_ids: Sequence[int],
        clock_ms: float,
        eos_token_id: int | None = None,
        stop_on_eos: bool = True,
        states: Sequence[RequestState] | None = None,
    ) -> list[RequestState]:
        targets = self._running if states is None else states
        return [s for s, t in zip(targets, token_ids) if s.append_token(t, clock_ms, eos_token_id, stop_on_eos)]

    def retire(self, finished: Sequence[RequestState]) -> None:
        for s in finished:
            s.status = RequestStatus.FINISHED
            assert s.batch_slot_idx is not None
            heapq.heappush(self._free_slots, s.batch_slot_idx)
        self._running = [s for s in self._running if s.status is RequestStatus.RUNNING]


def prepare_schedule(
    requests: Sequence[Request], max_running_requests: int
) -> tuple[list[RequestState], ArrivalQueue, float]:
    if max_running_requests < 1:
        raise ValueError("max_running_requests must be positive")
    validate_requests(requests)
    states = [RequestState(r) for r in requests]
    return states, ArrivalQueue(states), min(s.request.arrival_ms for s in states)


class SchedulePhase(str, Enum):
    PREFILL = "prefill"
    DECODE = "decode"
    MIXED = "mixed"  # decode rows and prefill chunks in one step (ChunkedPrefillConfig(mixed=True))

    def __str__(self) -> str:
        return self.value


@dataclass(frozen=True)
class PrefillChunk:
    """Prompt interval [start, end) of one request prefilled in one step; start = tokens already cached."""

    state: RequestState
    start: int
    end: int

    @property
    def num_tokens(self) -> int:
        return self.end - self.start

    @property
    def is_last(self) -> bool:
        return self.end == self.state.request.prompt_len


@dataclass(frozen=True)
class SchedulerOutput:
    """One step's decision.  num_scheduled_tokens: padded chunk tokens (prefill) or rows (decode);
    a mixed step has its decode rows in ``scheduled_requests`` and counts rows + padded chunk tokens."""

    phase: SchedulePhase
    scheduled_requests: tuple[RequestState, ...]
    num_scheduled_tokens: int
    is_oversize_prefill: bool = False
    prefill_chunks: tuple[PrefillChunk, ...] = ()


def _whole_prompts(states: Sequence[RequestState]) -> tuple[PrefillChunk, ...]:
    return tuple(PrefillChunk(s, 0, s.request.prompt_len) for s in states)


def _fit_budget(candidates: tuple[RequestState, ...], token_budget: int) -> tuple[tuple[RequestState, ...], bool]:
    """Longest FCFS prefix whose padded size fits; a head request alone over budget runs alone."""
    taken, longest = 0, 0
    for s in candidates:
        widest = max(longest, s.request.prompt_len)
        if (taken + 1) * widest > token_budget:
            break
        taken, longest = taken + 1, widest
    if taken == 0:
        return candidates[:1], True
    return candidates[:taken], False


class IterationScheduler:
    def __init__(
        self,
        scheduler_config: SchedulerConfig,
        batching_method: BatchingMethod,
        kv_cache_manager: KVCacheManager | None = None,
    ) -> None:
        if scheduler_config.max_running_requests is None:
            raise ValueError("scheduler_config.max_running_requests must be resolved to a positive int")
        self.scheduler_config = scheduler_config
        self.batching_method = batching_method
        self.waiting_queue = WaitingQueue()
        self.running_queue = RunningQueue(scheduler_config.max_running_requests)
        self.kv_cache_manager = kv_cache_manager
        self._last_phase: SchedulePhase | None = None

    @property
    def has_unfinished_requests(self) -> bool:
        return bool(self.waiting_queue or self.running_queue)

    def add_requests(self, states: Iterable[RequestState]) -> None:
        self.waiting_queue.extend(states)

    def schedule(self, clock_ms: float) -> SchedulerOutput | None:
        out = self._decide()
        if out is None:
            return None
        if out.phase is not SchedulePhase.DECODE:
            newcomers = sum(1 for c in out.prefill_chunks if c.state.status is RequestStatus.WAITING)
            self.running_queue.admit(self.waiting_queue.pop_batch(newcomers), clock_ms)
            for c in out.prefill_chunks:
                self._allocate_slots(c.state, c.num_tokens)
        if out.phase is not SchedulePhase.PREFILL:
            for s in out.scheduled_requests:
                self._allocate_slots(s, 1)
        self._last_phase = out.phase
        return out

    def update_from_output(
        self,
        scheduler_output: SchedulerOutput,
        token_ids: Sequence[int],
        clock_ms: float,
        eos_token_id: int | None = None,
        stop_on_eos: bool = True,
    ) -> list[RequestState]:
        if scheduler_output.phase is SchedulePhase.DECODE:
            for s in scheduler_output.scheduled_requests:
                s.cache_length += 1
            producers = scheduler_output.scheduled_requests
        elif scheduler_output.phase is SchedulePhase.PREFILL:
            for c in scheduler_output.prefill_chunks:
                c.state.cache_length = c.end
            producers = tuple(c.state for c in scheduler_output.prefill_chunks if c.is_last)
        else:  # mixed: token_ids = one per decode row, then one per chunk that ends its prompt
            for s in scheduler_output.scheduled_requests:
                s.cache_length += 1
            for c in scheduler_output.prefill_chunks:
                c.state.cache_length = c.end
            producers = (*scheduler_output.scheduled_requests,
                         *(c.state for c in scheduler_output.prefill_chunks if c.is_last))
        finished = self.running_queue.process_step_output(token_ids, clock_ms, eos_token_id, stop_on_eos, producers)
        if finished:
            if self.kv_cache_manager is not None:
                for s in finished:
                    self.kv_cache_manager.free(s.request.request_idx)
            self.running_queue.retire(finished)
        return finished

    def _allocate_slots(self, state: RequestState, num_new_tokens: int) -> None:
        if self.kv_cache_manager is None:
            return
        if not self.kv_cache_manager.allocate_slots(state.request.request_idx, num_new_tokens):
            raise RuntimeError("paged KV cache out of blocks (物理块已耗尽; there is no preemption): increase num_blocks")

    def _reserved_blocks(self) -> int:
        assert self.kv_cache_manager is not None
        bs = self.kv_cache_manager.block_size
        return sum(
            num_blocks_for_tokens(s.request.prompt_len, bs) - num_blocks_for_tokens(s.cache_length, bs)
            for s in self.running_queue.prefilling_requests
        )

    def _admission_candidates(self) -> tuple[RequestState, ...]:
        continuous = self.batching_method is BatchingMethod.CONTINUOUS
        if not (self.running_queue.can_admit() if continuous else not self.running_queue):
            return ()
        candidates = self.waiting_queue.requests[: self.running_queue.num_free_batch_slots]
        if self.kv_cache_manager is not None:
            fit = self.kv_cache_manager.num_admissible([s.request.prompt_len for s in candidates],
                                                       self._reserved_blocks())
            candidates = candidates[:fit]
        return candidates

    def _prefill(self, chunks: tuple[PrefillChunk, ...], oversize: bool = False) -> SchedulerOutput:
        return SchedulerOutput(
            phase=SchedulePhase.PREFILL,
            scheduled_requests=tuple(c.state for c in chunks),
            num_scheduled_tokens=len(chunks) * max(c.num_tokens for c in chunks),
            is_oversize_prefill=oversize,
            prefill_chunks=chunks,
        )

    def _decode(self) -> SchedulerOutput:
        rows = self.running_queue.decoding_requests
        return SchedulerOutput(phase=SchedulePhase.DECODE, scheduled_requests=rows, num_scheduled_tokens=len(rows))

    def _plan_chunks(self, token_budget: int, limit: int | None = None) -> tuple[PrefillChunk, ...]:
        candidates = (*self.running_queue.prefilling_requests, *self._admission_candidates())
        if limit is not None:
            candidates = candidates[:limit]
        if not candidates:
            return ()
        cap = token_budget // len(candidates)
        return tuple(
            PrefillChunk(s, s.cache_length, s.cache_length + min(s.request.prompt_len - s.cache_length, cap))
            for s in candidates
        )

    def _decide(self) -> SchedulerOutput | None:
        policy = self.scheduler_config.batching_policy
        if isinstance(policy, ChunkedPrefillConfig) and policy.mixed:
            rows = self.running_queue.decoding_requests
            budget = policy.token_budget - len(rows)
            chunks = self._plan_chunks(budget, limit=budget) if budget > 0 else ()
            if chunks and rows:
                return SchedulerOutput(
                    phase=SchedulePhase.MIXED, scheduled_requests=rows,
                    num_scheduled_tokens=len(rows) + len(chunks) * max(c.num_tokens for c in chunks),
                    prefill_chunks=chunks,
                )
            if chunks:
                return self._prefill(chunks)
            return self._decode() if rows else None
        if isinstance(policy, ChunkedPrefillConfig):
            if self.running_queue.decoding_requests and self._last_phase is SchedulePhase.PREFILL:
                return self._decode()
            chunks = self._plan_chunks(policy.token_budget)
            if chunks:
                return self._prefill(chunks)
            return self._decode() if self.running_queue.decoding_requests else None
        candidates = self._admission_candidates()
        if isinstance(policy, PrefillFirstConfig):
            if candidates:
                return self._prefill(_whole_prompts(candidates))
            return self._decode() if self.running_queue else None
        if self.running_queue and self._last_phase is SchedulePhase.PREFILL:
            return self._decode()
        if candidates:
            chosen, oversize = _fit_budget(candidates, policy.token_budget)
            return self._prefill(_whole_prompts(chosen), oversize)
        return self._decode() if self.running_queue else None
