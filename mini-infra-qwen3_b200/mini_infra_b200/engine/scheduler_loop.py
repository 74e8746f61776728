"""Engine loop (reference ``engine/scheduler_loop.py``) for the paged KV cache.

Arrivals move into the scheduler when the logical clock passes them; each iteration schedules one
prefill or decode step, runs it on the backend, advances the clock by the step's measured
model_ms + cache_ms, and feeds the tokens back.  With a head-partitioned model (several ranks)
every rank runs this loop; rank 0's measured step time is broadcast so that all ranks' clocks,
and hence their schedules and collectives, stay identical.
"""

from __future__ import annotations

import time
from collections.abc import Sequence

import torch

from mini_infra_b200.core import IterationScheduler, NoCacheConfig, PagedCacheConfig, Request, SchedulePhase
from mini_infra_b200.core import prepare_schedule
from mini_infra_b200.core.types import BatchingMethod
from mini_infra_b200.device import synchronize
from mini_infra_b200.engine.config import EngineConfig, validate_engine_config
from mini_infra_b200.engine.metrics import ScheduleEvent, ScheduleResult, summarize_schedule
from mini_infra_b200.engine.paged_schedule_backend import PagedScheduleBackend


def _shared_step_ms(step_ms: float, model: torch.nn.Module, device: torch.device) -> float:
    part = getattr(model, "partition", None)
    if part is None or part.world == 1:
        return step_ms
    import torch.distributed as dist

    t = torch.tensor([step_ms], dtype=torch.float64, device=device)
    dist.broadcast(t, src=dist.get_global_rank(part.group, 0) if part.group is not None else 0, group=part.group)
    return float(t.item())


@torch.inference_mode()
def _run_loop(backend: PagedScheduleBackend, requests: Sequence[Request], max_running_requests: int,
              config: EngineConfig, eos_token_id: int | None, stop_on_eos: bool) -> ScheduleResult:
    states, arrivals, clock_ms = prepare_schedule(requests, max_running_requests)
    scheduler = IterationScheduler(config.scheduler_config.with_max_running_requests(max_running_requests),
                                   backend.batching_method, backend.kv_cache_manager)
    events: list[ScheduleEvent] = []
    wall0 = time.perf_counter()
    pending_sched_ms = 0.0
    while arrivals or scheduler.has_unfinished_requests:
        t0 = time.perf_counter()
        scheduler.add_requests(arrivals.pop_arrived(clock_ms))
        out = scheduler.schedule(clock_ms)
        pending_sched_ms += (time.perf_counter() - t0) * 1000.0
        if out is None:
            clock_ms = arrivals.next_arrival_ms()
            continue
        active = len(scheduler.running_queue)
        if out.phase is SchedulePhase.PREFILL:
            step = backend.execute_prefill(out.prefill_chunks)
            admitted = tuple(c.state.request.request_idx for c in out.prefill_chunks if c.start == 0)
        elif out.phase is SchedulePhase.MIXED:
            step = backend.execute_mixed(out.scheduled_requests, out.prefill_chunks)
            admitted = tuple(c.state.request.request_idx for c in out.prefill_chunks if c.start == 0)
        else:
            step = backend.execute_decode(out.scheduled_requests)
            admitted = ()
        step_ms = _shared_step_ms(step.model_ms + step.cache_ms, backend.model, backend.device)
        clock_ms += step_ms
        t1 = time.perf_counter()
        finished = scheduler.update_from_output(out, step.next_tokens, clock_ms, eos_token_id, stop_on_eos)
        sched_ms = pending_sched_ms + (time.perf_counter() - t1) * 1000.0
        pending_sched_ms = 0.0
        backend.retire(finished, is_idle=not scheduler.running_queue)
        events.append(ScheduleEvent(
            phase=out.phase, admitted_request_ids=admitted,
            finished_request_ids=tuple(s.request.request_idx for s in finished),
            physical_batch_size=step.physical_batch_size, num_active_requests=active,
            num_generated_tokens=len(step.next_tokens), num_scheduled_tokens=out.num_scheduled_tokens,
            step_ms=step_ms, model_ms=step.model_ms, cache_management_ms=step.cache_ms, scheduler_ms=sched_ms,
            live_kv_cache_bytes=step.live_kv_cache_bytes, kv_cache_pool_bytes=step.kv_cache_pool_bytes,
            accessed_kv_cache_tokens=step.accessed_kv_cache_tokens, is_oversize_prefill=out.is_oversize_prefill,
        ))
    synchronize(backend.device)
    wall_ms = (time.perf_counter() - wall0) * 1000.0
    dev = backend.device
    cuda = dev.type == "cuda"
    result = summarize_schedule(
        states, events, max_running_requests, wall_ms, backend.collect_paged_cache_profile(),
        batching_method=backend.batching_method, kv_cache_config=backend.kv_cache_config,
        peak_allocated_mb=torch.cuda.max_memory_allocated(dev) / 1024**2 if cuda else 0.0,
        peak_reserved_mb=torch.cuda.max_memory_reserved(dev) / 1024**2 if cuda else 0.0,
        baseline_mb=backend.baseline_mb, is_cuda=cuda)
    result.extra.update(h2d_bytes=backend.runner.h2d_bytes, d2h_bytes=backend.runner.d2h_bytes,
                        decode_graph_replays=backend.runner.graph_replays,
                        mixed_graph_replays=backend.runner.mixed_graph_replays,
                        prefill_graph_replays=backend.runner.prefill_graph_replays)
    return result


@torch.inference_mode()
def run_scheduler(
    config: EngineConfig,
    model: torch.nn.Module,
    requests: Sequence[Request],
    eos_token_id: int | None = None,
    *,
    pad_token_id: int = 0,
    stop_on_eos: bool = True,
    cuda_graphs: bool = True,
    peer_exchange: bool = True,
) -> ScheduleResult:
    """Run the requests through the paged engine; returns sequences, events and metrics.

    ``cuda_graphs`` replays decode steps from per-batch-bucket CUDA graphs and prefill and mixed
    steps from per-shape graphs (False: eager).
    ``peer_exchange`` (head-partitioned bf16/fp16 models): decode outputs are exchanged by the
    decode kernel's peer stores (``exchange.PeerExchange``); False keeps the NCCL all-gather."""
    if not requests:
        raise ValueError("requests must not be empty")
    mrr = config.scheduler_config.max_running_requests or len(requests)
    if isinstance(config.kv_cache_config, NoCacheConfig):
        raise ValueError("the scheduler needs a KV cache")
    validate_engine_config(config.with_max_running_requests(mrr))
    if not isinstance(config.kv_cache_config, PagedCacheConfig):
        raise NotImplementedError("only caching-method=paged-kv-cache is implemented in this package")
    if config.batching_method not in (BatchingMethod.CONTINUOUS, BatchingMethod.FIXED):
        raise ValueError(f"paged-kv-cache supports continuous or fixed batching, got {config.batching_method.value}")
    backend = PagedScheduleBackend(model, requests, mrr, config.kv_cache_config, config.batching_method, pad_token_id,
                                   cuda_graphs=cuda_graphs, peer_exchange=peer_exchange)
    try:
        return _run_loop(backend, requests, mrr, config, eos_token_id, stop_on_eos)
    finally:
        backend.close()
