"""Control-plane configuration and result types (no torch).

Mirrors the reference's ``core/types.py`` (``PagedCacheConfig`` at core/types.py:47-66,
``ChunkedPrefillConfig``, ``SchedulerConfig``, ``BatchingMethod``, the string parsers) so that
configuration code written for the reference runs unchanged.  Only the kinds the paged path
needs are accepted; ``dense-kv-cache`` parses (for config compatibility) but the engine here
runs the paged path only.
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass, replace
from enum import Enum
from typing import Any, ClassVar, Literal

KVCacheKind = Literal["none", "dense-kv-cache", "paged-kv-cache"]
KV_CACHE_KINDS: tuple[KVCacheKind, ...] = ("none", "dense-kv-cache", "paged-kv-cache")

BatchingPolicyKind = Literal["prefill-first", "token-budget", "chunked-prefill"]
BATCHING_POLICY_KINDS: tuple[BatchingPolicyKind, ...] = ("prefill-first", "token-budget", "chunked-prefill")


def parse_kv_cache_kind(value: str | None) -> KVCacheKind:
    if value is None:
        return "none"
    if value in KV_CACHE_KINDS:
        return value  # type: ignore[return-value]
    raise ValueError(f"unknown KV cache kind {value!r}; choose one of {list(KV_CACHE_KINDS)}")


def parse_batching_policy_kind(value: str | None) -> BatchingPolicyKind:
    if value is None:
        return "prefill-first"
    if value in BATCHING_POLICY_KINDS:
        return value  # type: ignore[return-value]
    raise ValueError(f"unknown batching policy {value!r}; choose one of {list(BATCHING_POLICY_KINDS)}")


@dataclass(frozen=True)
class NoCacheConfig:
    kind: ClassVar[KVCacheKind] = "none"

    def __str__(self) -> str:
        return "no-cache"


@dataclass(frozen=True)
class DenseCacheConfig:
    kind: ClassVar[KVCacheKind] = "dense-kv-cache"

    def __str__(self) -> str:
        return self.kind


@dataclass(frozen=True)
class PagedCacheConfig:
    """Paged KV cache: tokens per block, and the pool size in blocks including the null block
    (None = derived from the workload by ``required_pool_blocks``)."""

    kind: ClassVar[KVCacheKind] = "paged-kv-cache"
    block_size: int = 16
    num_blocks: int | None = None

    def __post_init__(self) -> None:
        if self.block_size < 1:
            raise ValueError("block_size must be positive")
        if self.num_blocks is not None and self.num_blocks < 2:
            raise ValueError("num_blocks must be >= 2 (block 0 is the null block)")

    def __str__(self) -> str:
        extra = f",num_blocks={self.num_blocks}" if self.num_blocks is not None else ""
        return f"{self.kind}(block_size={self.block_size}{extra})"


KVCacheConfig = NoCacheConfig | DenseCacheConfig | PagedCacheConfig


def kv_cache_config_from_str(
    kind: str | None, *, block_size: int | None = None, num_blocks: int | None = None
) -> KVCacheConfig:
    parsed = parse_kv_cache_kind(kind)
    if parsed == "none":
        return NoCacheConfig()
    if parsed == "dense-kv-cache":
        return DenseCacheConfig()
    return PagedCacheConfig(block_size=16 if block_size is None else block_size, num_blocks=num_blocks)


def _positive_budget(budget: int) -> None:
    if budget < 1:
        raise ValueError("token_budget must be positive")


@dataclass(frozen=True)
class PrefillFirstConfig:
    """Admit every admissible waiting request as one whole-prompt prefill before decoding."""

    kind: ClassVar[BatchingPolicyKind] = "prefill-first"

    def __str__(self) -> str:
        return self.kind


@dataclass(frozen=True)
class TokenBudgetConfig:
    """Whole-prompt prefills limited to ``token_budget`` padded tokens (soft), with decode protection."""

    kind: ClassVar[BatchingPolicyKind] = "token-budget"
    token_budget: int

    def __post_init__(self) -> None:
        _positive_budget(self.token_budget)

    def __str__(self) -> str:
        return f"{self.kind}(token_budget={self.token_budget})"


@dataclass(frozen=True)
class ChunkedPrefillConfig:
    """Prompts are cut into chunks; one prefill step never exceeds ``token_budget`` padded tokens.

    ``mixed`` (no counterpart in the reference, whose chunked prefill alternates prefill and
    decode steps): every step carries all decoding requests, one token each, plus prefill chunks
    cut from what is left of the budget (``token_budget`` minus the decode rows), in one model
    forward.  Off by default, so schedules match the reference's."""

    kind: ClassVar[BatchingPolicyKind] = "chunked-prefill"
    token_budget: int
    mixed: bool = False

    def __post_init__(self) -> None:
        _positive_budget(self.token_budget)

    def __str__(self) -> str:
        return f"{self.kind}(token_budget={self.token_budget}{', mixed' if self.mixed else ''})"


BatchingPolicy = PrefillFirstConfig | TokenBudgetConfig | ChunkedPrefillConfig
BudgetedBatchingPolicy = TokenBudgetConfig | ChunkedPrefillConfig


def batching_policy_from_str(kind: str | None, *, token_budget: int | None = None) -> BatchingPolicy:
    parsed = parse_batching_policy_kind(kind)
    if parsed == "prefill-first":
        return PrefillFirstConfig()
    if token_budget is None:
        raise ValueError(f"{parsed} needs a token_budget")
    return ChunkedPrefillConfig(token_budget) if parsed == "chunked-prefill" else TokenBudgetConfig(token_budget)


@dataclass(frozen=True)
class SchedulerConfig:
    """Iteration scheduler knobs: concurrency cap (None = number of requests) and batching policy."""

    max_running_requests: int | None = None
    batching_policy: BatchingPolicy = PrefillFirstConfig()

    def __post_init__(self) -> None:
        if self.max_running_requests is not None and self.max_running_requests < 1:
            raise ValueError(f"max_running_requests must be positive, got {self.max_running_requests}")

    def with_max_running_requests(self, max_running_requests: int | None) -> "SchedulerConfig":
        return replace(self, max_running_requests=max_running_requests)

    def with_batching_policy(self, batching_policy: BatchingPolicy) -> "SchedulerConfig":
        return replace(self, batching_policy=batching_policy)

    def __str__(self) -> str:
        if self.max_running_requests is None:
            return str(self.batching_policy)
        return f"mrr={self.max_running_requests}+{self.batching_policy}"


def scheduler_config_from_str(
    kind: str | None = None, *, max_running_requests: int | None = None, token_budget: int | None = None
) -> SchedulerConfig:
    return SchedulerConfig(max_running_requests, batching_policy_from_str(kind, token_budget=token_budget))


class BatchingMethod(str, Enum):
    NONE = "none"
    FIXED = "fixed-batching"
    CONTINUOUS = "continuous-batching"

    @classmethod
    def from_str(cls, value: "str | BatchingMethod | None") -> "BatchingMethod":
        if value is None:
            return cls.NONE
        if isinstance(value, cls):
            return value
        try:
            return cls(value)
        except ValueError as err:
            raise ValueError(f"unknown batching method {value!r}; choose one of {[m.value for m in cls]}") from err

    def __str__(self) -> str:
        return self.value


@dataclass(frozen=True)
class SequenceOutput:
    request_idx: int
    token_ids: list[int]
    prompt_len: int
    output_len: int
    finish_reason: str
    completion_step: int | None = None


@dataclass(frozen=True)
class RequestMetrics:
    request_idx: int
    arrival_ms: float
    admitted_ms: float
    first_token_ms: float
    completion_ms: float
    num_output_tokens: int
    token_times_ms: tuple[float, ...]

    @property
    def queue_ms(self) -> float:
        return self.admitted_ms - self.arrival_ms

    @property
    def ttft_ms(self) -> float:
        return self.first_token_ms - self.arrival_ms

    @property
    def end_to_end_ms(self) -> float:
        return self.completion_ms - self.arrival_ms

    @property
    def inter_token_latencies_ms(self) -> list[float]:
        t = self.token_times_ms
        return [b - a for a, b in zip(t, t[1:])]


def collapse_uniform(values: Sequence[Any]) -> Any:
    if not values:
        return ()
    return values[0] if all(v == values[0] for v in values) else tuple(values)
