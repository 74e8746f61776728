"""Control plane of the paged path (pure CPU, no torch): requests, queues, scheduler, block tables."""

from mini_infra_b200.core.block_manager import (
    NULL_BLOCK_ID,
    FreeKVCacheBlockQueue,
    KVCacheManager,
    num_blocks_for_tokens,
    required_pool_blocks,
)
from mini_infra_b200.core.request import Request, RequestState, RequestStatus, make_requests, validate_requests
from mini_infra_b200.core.scheduler import (
    ArrivalQueue,
    IterationScheduler,
    PrefillChunk,
    RunningQueue,
    SchedulePhase,
    SchedulerOutput,
    WaitingQueue,
    prepare_schedule,
)
from mini_infra_b200.core.types import (
    BATCHING_POLICY_KINDS,
    KV_CACHE_KINDS,
    BatchingMethod,
    BatchingPolicy,
    BatchingPolicyKind,
    BudgetedBatchingPolicy,
    ChunkedPrefillConfig,
    DenseCacheConfig,
    KVCacheConfig,
    KVCacheKind,
    NoCacheConfig,
    PagedCacheConfig,
    PrefillFirstConfig,
    RequestMetrics,
    SchedulerConfig,
    SequenceOutput,
    TokenBudgetConfig,
    batching_policy_from_str,
    collapse_uniform,
    kv_cache_config_from_str,
    parse_batching_policy_kind,
    parse_kv_cache_kind,
    scheduler_config_from_str,
)

__all__ = [name for name in dir() if not name.startswith("_")]
