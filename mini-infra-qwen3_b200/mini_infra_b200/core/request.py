"""Requests and their mutable scheduling state (no torch).

Same contract as the reference's ``core/request.py``: ``Request`` is an immutable payload on a
logical timeline, ``RequestState`` tracks admission, the KV tokens already cached
(``cache_length``, advanced per chunk and per decode step) and the generated tokens.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass, field
from enum import Enum
from typing import Any

from mini_infra_b200.core.types import RequestMetrics, SequenceOutput


class RequestStatus(str, Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"

    def __str__(self) -> str:
        return self.value


@dataclass(frozen=True)
class Request:
    request_idx: int
    token_ids: tuple[int, ...]
    max_new_tokens: int
    arrival_ms: float = 0.0

    def __post_init__(self) -> None:
        if self.request_idx < 0:
            raise ValueError("request_idx must be >= 0")
        if not self.token_ids:
            raise ValueError("prompt must not be empty")
        if self.max_new_tokens < 1:
            raise ValueError("max_new_tokens must be >= 1")
        if self.arrival_ms < 0:
            raise ValueError("arrival_ms must be >= 0")

    @property
    def prompt_len(self) -> int:
        return len(self.token_ids)


def _stamp(value: float | None, name: str, request_idx: int) -> float:
    if value is None:
        raise RuntimeError(f"request {request_idx} has no {name}: it never completed")
    return value


@dataclass
class RequestState:
    request: Request
    status: RequestStatus = RequestStatus.WAITING
    generated: list[int] = field(default_factory=list)
    batch_slot_idx: int | None = None
    cache_length: int = 0  # tokens whose K/V are (scheduled to be) in the cache
    admitted_ms: float | None = None
    first_token_ms: float | None = None
    completion_ms: float | None = None
    token_times_ms: list[float] = field(default_factory=list)
    finish_reason: str = "max_tokens"

    @property
    def is_prefilling(self) -> bool:
        """Admitted, but part of the prompt is still missing from the cache (chunked prefill)."""
        return self.status is RequestStatus.RUNNING and self.cache_length < self.request.prompt_len

    def append_token(
        self, token_id: int, timestamp_ms: float, eos_token_id: int | None = None, stop_on_eos: bool = True
    ) -> bool:
        """Record one generated token; True when the request has finished (EOS or budget)."""
        self.generated.append(token_id)
        self.token_times_ms.append(timestamp_ms)
        if self.first_token_ms is None:
            self.first_token_ms = timestamp_ms
        hit_eos = stop_on_eos and eos_token_id is not None and token_id == eos_token_id
        if hit_eos or len(self.generated) >= self.request.max_new_tokens:
            self.completion_ms = timestamp_ms
            self.finish_reason = "stop" if hit_eos else "max_tokens"
            return True
        return False

    def to_sequence_output(self, completion_step: int | None = None) -> SequenceOutput:
        return SequenceOutput(
            request_idx=self.request.request_idx,
            token_ids=list(self.generated),
            prompt_len=self.request.prompt_len,
            output_len=len(self.generated),
            finish_reason=self.finish_reason,
            completion_step=completion_step,
        )

    def to_request_metrics(self) -> RequestMetrics:
        idx = self.request.request_idx
        return RequestMetrics(
            request_idx=idx,
            arrival_ms=self.request.arrival_ms,
            admitted_ms=_stamp(self.admitted_ms, "admitted_ms", idx),
            first_token_ms=_stamp(self.first_token_ms, "first_token_ms", idx),
            completion_ms=_stamp(self.completion_ms, "completion_ms", idx),
            num_output_tokens=len(self.generated),
            token_times_ms=tuple(self.token_times_ms),
        )


def make_requests(
    token_sequences: Sequence[Any],
    max_new_tokens: int | Sequence[int],
    arrival_times_ms: Sequence[float] | None = None,
) -> list[Request]:
    """Build requests numbered in submission order."""
    prompts = [tuple(int(t) for t in seq) for seq in token_sequences]
    budgets = [max_new_tokens] * len(prompts) if isinstance(max_new_tokens, int) else list(max_new_tokens)
    arrivals = [0.0] * len(prompts) if arrival_times_ms is None else list(arrival_times_ms)
    if not (len(budgets) == len(prompts) == len(arrivals)):
        raise ValueError("prompts, budgets and arrival times must have the same length")
    return [Request(i, p, int(n), float(t)) for i, (p, n, t) in enumerate(zip(prompts, budgets, arrivals))]


def validate_requests(requests: Sequence[Request]) -> None:
    if not requests:
        raise ValueError("requests must not be empty")
    if len({r.request_idx for r in requests}) != len(requests):
        raise ValueError("request_idx values must be unique")
