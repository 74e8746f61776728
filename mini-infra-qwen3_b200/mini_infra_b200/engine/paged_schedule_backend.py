"""Paged backend (reference ``engine/paged_schedule_backend.py``): glues scheduler, runner and pool.

Per prefill step: chunk forward (model_ms, StepTimer), then ``store_prefill`` timed as cache_ms
(host wall clock between two synchronisations).  Per decode step: the step inputs built on the
device from the slot-indexed block-table mirror (``PagedRunner.prepare_decode_rows``: O(batch)
host work and upload) timed as cache_ms, then the decode forward (model_ms).  Per mixed step
(mixed chunked prefill): one forward over decode rows and chunks (model_ms), then the chunks'
``store_prefill`` as cache_ms.  Unless ``cuda_graphs=False``, decode steps replay a CUDA graph per
batch bucket, and prefill and mixed steps one graph per step shape holding forward + sample +
store (model_ms; cache_ms ~0; on a head partition they hold the NCCL all-gathers); a bucket's or
shape's first step captures its graph before the timing starts.  ``accessed_kv_cache_tokens``
counts history tokens read: sum of chunk starts (prefill) and sum of context lengths (decode).
"""

from __future__ import annotations

import time
from collections.abc import Sequence

import torch

from mini_infra_b200.core.block_manager import KVCacheManager, num_blocks_for_tokens, required_pool_blocks
from mini_infra_b200.core.request import Request, RequestState
from mini_infra_b200.core.scheduler import PrefillChunk
from mini_infra_b200.core.types import BatchingMethod, PagedCacheConfig
from mini_infra_b200.device import synchronize
from mini_infra_b200.engine.metrics import PagedCacheProfile
from mini_infra_b200.engine.schedule_backend import ScheduleStepOutput
from mini_infra_b200.worker import PagedKVCachePool, PagedRunner


class PagedScheduleBackend:
    def __init__(
        self,
        model: torch.nn.Module,
        requests: Sequence[Request],
        max_running_requests: int,
        paged_cache_config: PagedCacheConfig,
        batching_method: BatchingMethod = BatchingMethod.CONTINUOUS,
        pad_token_id: int = 0,
        cuda_graphs: bool = True,
        peer_exchange: bool = True,
    ) -> None:
        self.model = model
        self.device = next(model.parameters()).device
        # memory before the pool (the run's baseline), and peaks counted from here
        synchronize(self.device)
        self.baseline_mb = torch.cuda.memory_allocated(self.device) / 1024**2 if self.device.type == "cuda" else 0.0
        if self.device.type == "cuda":
            torch.cuda.reset_peak_memory_stats(self.device)
        self.max_running_requests = max_running_requests
        self.batching_method = batching_method
        self.paged_cache_config = paged_cache_config
        self.block_size = paged_cache_config.block_size
        num_blocks = paged_cache_config.num_blocks or required_pool_blocks(
            requests, max_running_requests, self.block_size)
        largest = max(num_blocks_for_tokens(r.prompt_len + r.max_new_tokens - 1, self.block_size) for r in requests)
        if largest > num_blocks - 1:
            raise ValueError(f"num_blocks={num_blocks} cannot hold one request's {largest} blocks (+1 null block)")
        config = model.config  # type: ignore[attr-defined]
        attn = model.model.layers[0].self_attn  # type: ignore[attr-defined]
        self.runner = PagedRunner(model, pad_token_id)
        self.pool = PagedKVCachePool(
            num_layers=config.num_hidden_layers,
            num_blocks=num_blocks,
            block_size=self.block_size,
            num_kv_heads=attn.num_kv_heads,
            head_dim=config.head_dim,
            dtype=next(model.parameters()).dtype,
            device=self.device,
        )
        self.kv_cache_manager = KVCacheManager(self.block_size, num_blocks)
        # decode inputs are built on the device from a slot-indexed mirror of the block tables
        self.runner.enable_device_tables(max_running_requests, largest)
        part = getattr(model, "partition", None)
        if part is not None and part.world > 1:
            # Decode outputs exchanged by peer stores, with rows for the largest decode step (kept on
            # the model across runs: detach_peer_exchange before the process group goes), or by
            # the NCCL all-gather (peer_exchange=False).
            from mini_infra_b200.exchange import attach_peer_exchange, detach_peer_exchange
            from mini_infra_b200.worker.decode_graphs import BUCKETS

            rows = max(max_running_requests, BUCKETS[-1])
            current = model.model.layers[0].self_attn.exchange  # type: ignore[attr-defined]
            if current is not None and (not peer_exchange or current.max_rows < rows):
                detach_peer_exchange(model)
                current = None
            if peer_exchange and current is None:
                attach_peer_exchange(model, rows, self.block_size)
        if cuda_graphs and self.device.type == "cuda":
            # decode tables never exceed the largest request; round the graphs' width up to a power of two
            width = 1 << max(4, (largest - 1).bit_length())
            self.runner.enable_decode_graphs(self.pool.kv_pools, width)
            self.runner.enable_mixed_graphs(self.pool, width)

    def close(self) -> None:
        """Drop the decode and mixed-step graphs (they may hold NCCL calls: before the process group goes)."""
        self.runner.release_decode_graphs()
        self.runner.release_mixed_graphs()

    @property
    def kv_cache_config(self) -> PagedCacheConfig:
        return self.paged_cache_config

    def execute_prefill(self, chunks: Sequence[PrefillChunk]) -> ScheduleStepOutput:
        tables = [self.kv_cache_manager.block_table(c.state.request.request_idx) for c in chunks]
        starts = [c.start for c in chunks]
        chunk_ids = [c.state.request.token_ids[c.start : c.end] for c in chunks]
        if self.runner.warm_mixed_graph([], chunk_ids, tables, self.pool):  # a shape's first step captures
            # a graph replay of forward + sample + the chunks' store (in model_ms)
            mixed = self.runner.run_mixed_step([], [], [], chunk_ids, starts, tables, self.pool)
            next_tokens, model_ms, cache = mixed.prefill_tokens, mixed.model_ms, None
        else:
            out = self.runner.run_prefill_chunk_step(chunk_ids, starts, tables, self.pool)
            next_tokens, model_ms, cache = out.next_tokens, out.model_ms, out.prefill_cache
        synchronize(self.device)
        t0 = time.perf_counter()
        if cache is not None:
            self.runner.store_prefill(self.pool, cache, tables, [c.num_tokens for c in chunks], starts)
        synchronize(self.device)
        cache_ms = (time.perf_counter() - t0) * 1000.0
        return ScheduleStepOutput(
            next_tokens=[t for t, c in zip(next_tokens, chunks) if c.is_last],
            model_ms=model_ms,
            cache_ms=cache_ms,
            physical_batch_size=len(chunks),
            live_kv_cache_bytes=self.kv_cache_manager.num_used_blocks * self.pool.bytes_per_block,
            kv_cache_pool_bytes=self.pool.total_bytes,
            accessed_kv_cache_tokens=sum(starts),
        )

    def execute_decode(self, scheduled: Sequence[RequestState]) -> ScheduleStepOutput:
        tables = [self.kv_cache_manager.block_table(s.request.request_idx) for s in scheduled]
        self.runner.warm_decode_graph(len(tables), max(len(t) for t in tables))  # first use of a bucket: capture
        synchronize(self.device)
        t0 = time.perf_counter()
        ids, pos, md = self.runner.prepare_decode_rows(
            [(s.batch_slot_idx, s.request.request_idx) for s in scheduled],
            tables,
            last_tokens=[s.generated[-1] for s in scheduled],
            positions=[s.cache_length for s in scheduled],
            block_size=self.block_size,
        )
        synchronize(self.device)
        cache_ms = (time.perf_counter() - t0) * 1000.0
        out = self.runner.run_decode_step(ids, pos, md, self.pool)
        return ScheduleStepOutput(
            next_tokens=out.next_tokens,
            model_ms=out.model_ms,
            cache_ms=cache_ms,
            physical_batch_size=len(scheduled),
            live_kv_cache_bytes=self.kv_cache_manager.num_used_blocks * self.pool.bytes_per_block,
            kv_cache_pool_bytes=self.pool.total_bytes,
            accessed_kv_cache_tokens=sum(s.cache_length + 1 for s in scheduled),
        )

    def execute_mixed(self, decoding: Sequence[RequestState], chunks: Sequence[PrefillChunk]) -> ScheduleStepOutput:
        """A mixed step (ChunkedPrefillConfig(mixed=True)): decode rows and prefill chunks in one
        forward, then ``store_prefill`` of the chunks (timed as cache_ms).  next_tokens: one per
        decode row, then one per chunk that ends its prompt."""
        d_tables = [self.kv_cache_manager.block_table(s.request.request_idx) for s in decoding]
        c_tables = [self.kv_cache_manager.block_table(c.state.request.request_idx) for c in chunks]
        starts = [c.start for c in chunks]
        chunk_ids = [c.state.request.token_ids[c.start : c.end] for c in chunks]
        self.runner.warm_mixed_graph(d_tables, chunk_ids, c_tables, self.pool)  # first use of a shape: capture
        out = self.runner.run_mixed_step(
            d_tables, [s.generated[-1] for s in decoding], [s.cache_length for s in decoding], chunk_ids, starts,
            c_tables, self.pool)
        synchronize(self.device)
        t0 = time.perf_counter()
        if out.prefill_cache is not None:  # None: a graph replay stored the chunks (in model_ms)
            self.runner.store_prefill(self.pool, out.prefill_cache, c_tables, [c.num_tokens for c in chunks], starts)
        synchronize(self.device)
        cache_ms = (time.perf_counter() - t0) * 1000.0
        return ScheduleStepOutput(
            next_tokens=out.decode_tokens + [t for t, c in zip(out.prefill_tokens, chunks) if c.is_last],
            model_ms=out.model_ms,
            cache_ms=cache_ms,
            physical_batch_size=len(decoding) + len(chunks),
            live_kv_cache_bytes=self.kv_cache_manager.num_used_blocks * self.pool.bytes_per_block,
            kv_cache_pool_bytes=self.pool.total_bytes,
            accessed_kv_cache_tokens=sum(starts) + sum(s.cache_length + 1 for s in decoding),
        )

    def retire(self, finished: Sequence[RequestState], *, is_idle: bool) -> None:
        return None

    def collect_paged_cache_profile(self) -> PagedCacheProfile:
        m = self.kv_cache_manager
        return PagedCacheProfile(self.block_size, self.pool.bytes_per_block, self.pool.num_blocks, m.peak_used_blocks,
                                 m.block_cold_allocation_count, m.block_reuse_count, m.block_release_count)
