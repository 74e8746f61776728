"""Requests and their scheduling state (pure Python: the control plane never imports torch).

What stays as in the reference's ``core/request.py``, because the scheduler, the engine and the
reference's own unit tests address it directly: the names ``Request`` / ``RequestState`` /
``RequestStatus`` / ``make_requests`` / ``validate_requests``, the fields of both dataclasses
(``cache_length`` counts the tokens whose K/V are scheduled into the cache: it advances by a
chunk per prefill step and by one per decode step), the finish reasons ``"stop"`` / ``"max_tokens"``
and the exception types.  Where the reference's tests match an error message, the message carries
the reference's wording in parentheses.

A request is finished by whichever comes first of EOS (when ``stop_on_eos``) and its token budget;
its timeline (admission, first token, completion, every token time) is stamped on the engine's
logical clock.
"""

from __future__ import annotations

import numbers
from collections import Counter
from collections.abc import Sequence
from dataclasses import dataclass, field
from enum import Enum
from typing import Any

from mini_infra_b200.core.types import RequestMetrics, SequenceOutput

STOP = "stop"  # finished on the EOS token
MAX_TOKENS = "max_tokens"  # finished on its token budget


class RequestStatus(str, Enum):
    WAITING = "waiting"
    RUNNING = "running"
    FINISHED = "finished"

    def __str__(self) -> str:
        return self.value


@dataclass(frozen=True)
class Request:
    """An immutable prompt with its output budget and its arrival time on the logical clock."""

    request_idx: int
    token_ids: tuple[int, ...]
    max_new_tokens: int
    arrival_ms: float = 0.0

    def __post_init__(self) -> None:
        checks = (
            (self.request_idx < 0, f"request_idx must not be negative (got {self.request_idx})"),
            (len(self.token_ids) == 0, "the prompt must hold at least one token"),
            (self.max_new_tokens < 1, f"max_new_tokens must be at least 1 (got {self.max_new_tokens})"),
            (self.arrival_ms < 0, f"arrival_ms must not be negative (got {self.arrival_ms})"),
        )
        problems = [message for failed, message in checks if failed]
        if problems:
            raise ValueError("; ".join(problems))

    @property
    def prompt_len(self) -> int:
        return len(self.token_ids)


@dataclass
class RequestState:
    """The mutable side of a request while the scheduler holds it."""

    request: Request
    status: RequestStatus = RequestStatus.WAITING
    generated: list[int] = field(default_factory=list)
    batch_slot_idx: int | None = None
    cache_length: int = 0
    admitted_ms: float | None = None
    first_token_ms: float | None = None
    completion_ms: float | None = None
    token_times_ms: list[float] = field(default_factory=list)
    finish_reason: str = MAX_TOKENS

    @property
    def is_prefilling(self) -> bool:
        """Admitted, with part of the prompt not yet in the cache (between chunks of a chunked prefill)."""
        return self.status is RequestStatus.RUNNING and self.cache_length < self.request.prompt_len

    def _reason_to_finish(self, token_id: int, eos_token_id: int | None, stop_on_eos: bool) -> str | None:
        if stop_on_eos and eos_token_id is not None and token_id == eos_token_id:
            return STOP
        if len(self.generated) >= self.request.max_new_tokens:
            return MAX_TOKENS
        return None

    def append_token(
        self, token_id: int, timestamp_ms: float, eos_token_id: int | None = None, stop_on_eos: bool = True
    ) -> bool:
        """Record one generated token at `timestamp_ms`; True once the request is finished."""
        self.generated.append(token_id)
        self.token_times_ms.append(timestamp_ms)
        self.first_token_ms = self.token_times_ms[0]
        reason = self._reason_to_finish(token_id, eos_token_id, stop_on_eos)
        if reason is None:
            return False
        self.finish_reason = reason
        self.completion_ms = timestamp_ms
        return True

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
        """The request's timeline; a request that never completed has none (RuntimeError)."""
        stamps = {"admitted_ms": self.admitted_ms, "first_token_ms": self.first_token_ms,
                  "completion_ms": self.completion_ms}
        missing = [name for name, value in stamps.items() if value is None]
        if missing:
            raise RuntimeError(f"request {self.request.request_idx} did not complete: no {', '.join(missing)}")
        return RequestMetrics(
            request_idx=self.request.request_idx,
            arrival_ms=self.request.arrival_ms,
            num_output_tokens=len(self.generated),
            token_times_ms=tuple(self.token_times_ms),
            **stamps,
        )


def _one_per_prompt(value: Any, count: int) -> list:
    """A scalar repeated for every prompt, or the sequence itself."""
    return [value] * count if isinstance(value, numbers.Real) else list(value)


def make_requests(
    token_sequences: Sequence[Any],
    max_new_tokens: int | Sequence[int],
    arrival_times_ms: Sequence[float] | None = None,
) -> list[Request]:
    """Requests numbered in submission order: one budget for all or one per prompt, and arrival
    times (all 0 by default)."""
    prompts = [tuple(int(t) for t in seq) for seq in token_sequences]
    budgets = _one_per_prompt(max_new_tokens, len(prompts))
    arrivals = _one_per_prompt(0.0 if arrival_times_ms is None else arrival_times_ms, len(prompts))
    if len(budgets) != len(prompts) or len(arrivals) != len(prompts):
        raise ValueError(f"{len(prompts)} prompts, {len(budgets)} token budgets and {len(arrivals)} arrival times "
                         "(数量必须一致: the counts must agree)")
    return [Request(i, prompt, int(budget), float(arrival))
            for i, (prompt, budget, arrival) in enumerate(zip(prompts, budgets, arrivals))]


def validate_requests(requests: Sequence[Request]) -> None:
    """A workload is a non-empty list of requests with distinct ids (each request checks itself)."""
    if len(requests) == 0:
        raise ValueError("requests is empty (不能为空)")
    repeated = sorted(idx for idx, n in Counter(r.request_idx for r in requests).items() if n > 1)
    if repeated:
        raise ValueError(f"request_idx must be unique (唯一); repeated: {repeated}")


__all__ = ["Request", "RequestState", "RequestStatus", "make_requests", "validate_requests"]
