"""Engine configuration (reference ``engine/config.py``): KV cache kind, batching method,
scheduler config, and the validity rules of their combinations."""

from __future__ import annotations

from dataclasses import dataclass, replace

from mini_infra_b200.core.types import (
    BatchingMethod,
    BatchingPolicy,
    BudgetedBatchingPolicy,
    ChunkedPrefillConfig,
    KVCacheConfig,
    NoCacheConfig,
    PagedCacheConfig,
    PrefillFirstConfig,
    SchedulerConfig,
)


@dataclass(frozen=True)
class EngineConfig:
    kv_cache_config: KVCacheConfig = NoCacheConfig()
    batching_method: BatchingMethod = BatchingMethod.NONE
    flags: frozenset = frozenset()
    scheduler_config: SchedulerConfig = SchedulerConfig()

    def with_kv_cache_config(self, kv_cache_config: KVCacheConfig) -> "EngineConfig":
        return replace(self, kv_cache_config=kv_cache_config)

    def with_batching_method(self, batching_method: BatchingMethod) -> "EngineConfig":
        return replace(self, batching_method=batching_method)

    def with_scheduler_config(self, scheduler_config: SchedulerConfig) -> "EngineConfig":
        return replace(self, scheduler_config=scheduler_config)

    def with_max_running_requests(self, max_running_requests: int | None) -> "EngineConfig":
        return replace(self, scheduler_config=self.scheduler_config.with_max_running_requests(max_running_requests))

    def with_batching_policy(self, batching_policy: BatchingPolicy) -> "EngineConfig":
        return replace(self, scheduler_config=self.scheduler_config.with_batching_policy(batching_policy))

    @property
    def has_kv_cache(self) -> bool:
        return not isinstance(self.kv_cache_config, NoCacheConfig)

    @property
    def is_batch(self) -> bool:
        return self.batching_method != BatchingMethod.NONE

    def __str__(self) -> str:
        parts = [str(self.kv_cache_config)]
        if self.batching_method != BatchingMethod.NONE:
            parts.append(self.batching_method.value)
        if self.scheduler_config.max_running_requests is not None:
            parts.append(f"mrr={self.scheduler_config.max_running_requests}")
        if not isinstance(self.scheduler_config.batching_policy, PrefillFirstConfig):
            parts.append(str(self.scheduler_config.batching_policy))
        return "+".join(parts)


def validate_engine_config(config: EngineConfig) -> None:
    """Reject combinations the engine cannot run (same rules as the reference)."""
    if isinstance(config.kv_cache_config, PagedCacheConfig) and config.batching_method is BatchingMethod.NONE:
        raise ValueError("paged-kv-cache needs continuous-batching or fixed-batching")
    if config.batching_method is BatchingMethod.CONTINUOUS and isinstance(config.kv_cache_config, NoCacheConfig):
        raise ValueError("continuous-batching needs a KV cache")
    policy = config.scheduler_config.batching_policy
    if isinstance(policy, ChunkedPrefillConfig) and not isinstance(config.kv_cache_config, PagedCacheConfig):
        raise ValueError("chunked-prefill reads chunk history from the block pool: it needs paged-kv-cache")
    if isinstance(policy, BudgetedBatchingPolicy):
        if config.batching_method is not BatchingMethod.CONTINUOUS:
            raise ValueError(f"{policy.kind} needs continuous-batching, got {config.batching_method.value}")
        mrr = config.scheduler_config.max_running_requests
        if mrr is not None and policy.token_budget < mrr:
            raise ValueError(f"token_budget={policy.token_budget} must be >= max_running_requests={mrr}")
