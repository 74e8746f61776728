"""GPU data plane: physical block pools and the paged runner."""

from mini_infra_b200.worker.base_runner import BaseModelRunner, PrefillOutput
from mini_infra_b200.worker.kv_cache import KVCache, cache_size_bytes
from mini_infra_b200.worker.paged_kv_cache import PagedKVCachePool
from mini_infra_b200.worker.paged_runner import PagedDecodeOutput, PagedMixedOutput, PagedRunner
from mini_infra_b200.worker.sampler import greedy_sample

__all__ = [
    "BaseModelRunner",
    "KVCache",
    "PagedDecodeOutput",
    "PagedMixedOutput",
    "PagedKVCachePool",
    "PagedRunner",
    "PrefillOutput",
    "cache_size_bytes",
    "greedy_sample",
]
