"""The engine loop and its run summary on CPU, driven by a fake backend (no model, no GPU).

``_run_loop`` with this package's scheduler, block manager and ``summarize_schedule`` runs the
reference's schedules; the backend returns deterministic tokens and step times.  Checked:

* the summary equals the reference's own ``engine/metrics.py:summarize_schedule`` on the same
  request states and events, field by field (when the reference checkout is next to this
  repository; skipped elsewhere);
* the block-lifetime and timeline criteria of the reference's end-to-end paged scheduler tests
  (``tests/unit/test_paged_scheduler.py``, which need the reference's CPU engine and cannot run
  against this CUDA-only one), restated: every request admitted and finished once, event tokens
  summing to the outputs, decode steps without padding rows, live KV bytes a whole number of blocks
  and within the pool, admission gated by free blocks, EOS ending a request and freeing its blocks.
"""

import math
import os
import sys
from dataclasses import fields
from pathlib import Path
from types import SimpleNamespace

import pytest
import torch

from mini_infra_b200.core import (
    ChunkedPrefillConfig, KVCacheManager, PagedCacheConfig, PrefillFirstConfig, SchedulePhase, SchedulerConfig,
    TokenBudgetConfig, make_requests,
)
from mini_infra_b200.core.block_manager import required_pool_blocks
from mini_infra_b200.core.types import BatchingMethod
from mini_infra_b200.engine import EngineConfig, ScheduleStepOutput
from mini_infra_b200.engine.metrics import PagedCacheProfile, percentile
from mini_infra_b200.engine.scheduler_loop import _run_loop

ROOT = Path(__file__).resolve().parents[1]
REFERENCE = Path(os.environ.get("MINI_INFRA_REFERENCE", ROOT.parent / "reference"))
BLOCK_BYTES = 1024  # bytes of one block over all layers, K and V (any positive value)


def token_for(state) -> int:
    return (7 * state.request.request_idx + 3 * len(state.generated)) % 50 + 1


class FakeBackend:
    """The backend contract of PagedScheduleBackend without a model: tokens from ``token_for``,
    model_ms = 1 + 0.01 per token processed, cache_ms = 0.25, live bytes = used blocks."""

    def __init__(self, requests, mrr, block_size, num_blocks=None):
        self.model = SimpleNamespace()
        self.device = torch.device("cpu")
        self.batching_method = BatchingMethod.CONTINUOUS
        self.block_size = block_size
        self.num_blocks = num_blocks or required_pool_blocks(requests, mrr, block_size)
        self.kv_cache_manager = KVCacheManager(block_size, self.num_blocks)
        self.kv_cache_config = PagedCacheConfig(block_size, self.num_blocks)
        self.baseline_mb = 0.0
        self.runner = SimpleNamespace(h2d_bytes=0, d2h_bytes=0, graph_replays=0, mixed_graph_replays=0,
                                      prefill_graph_replays=0)
        self.used_blocks_seen = []

    def _out(self, tokens, n_tokens, rows, accessed):
        used = self.kv_cache_manager.num_used_blocks
        self.used_blocks_seen.append(used)
        return ScheduleStepOutput(next_tokens=tokens, model_ms=1.0 + 0.01 * n_tokens, cache_ms=0.25,
                                  physical_batch_size=rows, live_kv_cache_bytes=used * BLOCK_BYTES,
                                  kv_cache_pool_bytes=self.num_blocks * BLOCK_BYTES, accessed_kv_cache_tokens=accessed)

    def execute_prefill(self, chunks):
        tokens = [token_for(c.state) for c in chunks if c.is_last]
        return self._out(tokens, sum(c.num_tokens for c in chunks), len(chunks), sum(c.start for c in chunks))

    def execute_decode(self, scheduled):
        return self._out([token_for(s) for s in scheduled], len(scheduled), len(scheduled),
                         sum(s.cache_length + 1 for s in scheduled))

    def execute_mixed(self, decoding, chunks):
        tokens = [token_for(s) for s in decoding] + [token_for(c.state) for c in chunks if c.is_last]
        return self._out(tokens, len(decoding) + sum(c.num_tokens for c in chunks), len(decoding) + len(chunks),
                         sum(c.start for c in chunks))

    def retire(self, finished, *, is_idle):
        return None

    def collect_paged_cache_profile(self):
        m = self.kv_cache_manager
        return PagedCacheProfile(self.block_size, BLOCK_BYTES, self.num_blocks, m.peak_used_blocks,
                                 m.block_cold_allocation_count, m.block_reuse_count, m.block_release_count)


def prompts(lengths):
    return [[(i * 7 + j * 3) % 90 + 1 for j in range(n)] for i, n in enumerate(lengths)]


def run(lengths, budgets, policy, mrr, block_size=4, arrivals=None, num_blocks=None, eos=None):
    requests = make_requests(prompts(lengths), budgets, arrivals)
    backend = FakeBackend(requests, mrr, block_size, num_blocks)
    config = EngineConfig(PagedCacheConfig(block_size), BatchingMethod.CONTINUOUS, SchedulerConfig(mrr, policy))
    result = _run_loop(backend, requests, mrr, config, eos, eos is not None)
    return result, backend


CASES = {
    "prefill_first": ([4, 9, 6, 12, 3], [5, 3, 8, 2, 6], PrefillFirstConfig(), 3, [0.0, 0.0, 2.5, 7.0, 7.0]),
    "chunked": ([17, 5, 30, 8], [4, 6, 3, 5], ChunkedPrefillConfig(12), 2, [0.0, 1.0, 1.0, 40.0]),
    "token_budget": ([6, 14, 3, 9], [3, 4, 5, 2], TokenBudgetConfig(16), 3, None),
    "mixed": ([17, 5, 30, 8], [4, 6, 3, 5], ChunkedPrefillConfig(16, mixed=True), 3, [0.0, 1.0, 1.0, 2.0]),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_timeline_block_and_token_invariants(name):
    lengths, budgets, policy, mrr, arrivals = CASES[name]
    result, backend = run(lengths, budgets, policy, mrr, arrivals=arrivals)
    n = len(lengths)
    for r, budget in zip(result.request_metrics, budgets):
        assert r.arrival_ms <= r.admitted_ms <= r.first_token_ms <= r.completion_ms
        assert r.num_output_tokens == budget == len(r.token_times_ms)
    assert [s.token_ids for s in result.sequences] == [
        [(7 * i + 3 * k) % 50 + 1 for k in range(b)] for i, b in enumerate(budgets)]
    assert all(s.finish_reason == "max_tokens" for s in result.sequences)
    assert sum(e.num_generated_tokens for e in result.events) == sum(budgets)
    assert sorted(i for e in result.events for i in e.admitted_request_ids) == list(range(n))
    assert sorted(i for e in result.events for i in e.finished_request_ids) == list(range(n))
    decode = [e for e in result.events if e.phase is SchedulePhase.DECODE]
    assert all(e.physical_batch_size == e.num_active_requests for e in decode)  # no padding rows
    assert all(e.live_kv_cache_bytes % BLOCK_BYTES == 0 for e in result.events)
    assert max(e.live_kv_cache_bytes for e in result.events) <= (backend.num_blocks - 1) * BLOCK_BYTES
    assert backend.kv_cache_manager.num_used_blocks == 0  # every block released at the end
    assert result.schedule_metrics.busy_ms == pytest.approx(sum(e.step_ms for e in result.events))
    assert result.memory.kv_cache.peak_live_kv_cache_mb > 0
    assert result.batch_size == n and result.requests is result.request_metrics
    assert result.trace.step_latencies_ms == [e.step_ms for e in result.events]
    padded = result.padded_output_tokens()
    assert padded.shape == (n, max(budgets)) and padded[0, : budgets[0]].tolist() == result.sequences[0].token_ids


def test_live_bytes_peak_at_two_requests_of_three_blocks():
    # block size 4: 5-token prompts + 6 new tokens -> 10 cached tokens -> 3 blocks each, both at once
    result, _ = run([5, 5], [6, 6], PrefillFirstConfig(), 2, arrivals=[0.0, 0.0])
    assert max(e.live_kv_cache_bytes for e in result.events) == 6 * BLOCK_BYTES


def test_small_pool_gates_admission():
    # 3 requests of 6 + 3 tokens (2 blocks each at bs 4) in 1 null + 4 blocks: two run, one waits
    result, backend = run([6, 6, 6], [3, 3, 3], PrefillFirstConfig(), 3, num_blocks=5)
    prefill = [e for e in result.events if e.phase is SchedulePhase.PREFILL]
    assert [e.admitted_request_ids for e in prefill] == [(0, 1), (2,)]
    assert result.request_metrics[2].admitted_ms >= result.request_metrics[0].completion_ms
    assert max(backend.used_blocks_seen) <= 4


def test_eos_ends_a_request_and_frees_its_blocks():
    budgets = [8, 8, 8]
    eos = (7 * 0 + 3 * 2) % 50 + 1  # request 0's third token
    result, backend = run([4, 6, 5], budgets, PrefillFirstConfig(), 2, eos=eos)
    first = result.sequences[0]
    assert first.finish_reason == "stop" and first.token_ids[-1] == eos and len(first.token_ids) == 3
    assert backend.kv_cache_manager.num_used_blocks == 0


def test_percentile_is_nearest_rank():
    assert percentile([], 50) == 0.0
    assert percentile([3.0], 95) == 3.0
    values = [float(v) for v in range(1, 21)]
    assert percentile(values, 50) == 10.0 and percentile(values, 95) == 19.0 and percentile(values, 100) == 20.0
    assert percentile(values, 0) == 1.0
    assert percentile([5.0, 1.0, 3.0], 34) == 3.0  # ceil(3 * 0.34) = 2nd smallest


def _reference_summary(states, result, mrr):
    """The reference's summarize_schedule on the same states and events (its event type and enums)."""
    src = REFERENCE / "src"
    if not (src / "mini_infra" / "engine" / "metrics.py").exists():
        pytest.skip("no reference checkout next to this repository")
    if str(src) not in sys.path:
        sys.path.insert(0, str(src))
    from mini_infra.core.scheduler import SchedulePhase as RefPhase
    from mini_infra.core.types import BatchingMethod as RefBatching
    from mini_infra.engine import metrics as ref

    events = [ref.ScheduleEvent(**{f.name: (RefPhase[e.phase.name] if f.name == "phase" else getattr(e, f.name))
                                   for f in fields(ref.ScheduleEvent)}) for e in result.events]
    return ref.summarize_schedule(RefBatching.CONTINUOUS, states, events, mrr, 0.0, 0.0,
                                  e2e_wall_ms=result.e2e_wall_ms, is_cuda=False)


def _same(ours, theirs, where):
    for f in fields(theirs):
        a, b = getattr(ours, f.name), getattr(theirs, f.name)
        if isinstance(b, float) and isinstance(a, (int, float)):
            assert math.isclose(a, b, rel_tol=1e-12, abs_tol=1e-12), f"{where}.{f.name}: {a} != {b}"
        elif f.name != "paged_cache":
            assert a == b, f"{where}.{f.name}: {a} != {b}"


@pytest.mark.parametrize("name", ["prefill_first", "chunked", "token_budget"])
def test_summary_equals_the_references_summarize_schedule(name, monkeypatch):
    lengths, budgets, policy, mrr, arrivals = CASES[name]
    captured = {}
    import mini_infra_b200.engine.scheduler_loop as loop

    real = loop.summarize_schedule

    def keep_states(states, *a, **k):
        captured["states"] = list(states)
        return real(states, *a, **k)

    monkeypatch.setattr(loop, "summarize_schedule", keep_states)
    result, _ = run(lengths, budgets, policy, mrr, arrivals=arrivals)
    theirs = _reference_summary(captured["states"], result, mrr)
    _same(result.schedule_metrics, theirs.schedule_metrics, "schedule_metrics")
    _same(result.metrics, theirs.metrics, "metrics")
    _same(result.batch_info, theirs.batch_info, "batch_info")
    _same(result.memory.kv_cache, theirs.memory.kv_cache, "memory.kv_cache")
    assert result.trace.step_latencies_ms == theirs.trace.step_latencies_ms
    assert result.trace.num_active_tokens_per_step == theirs.trace.num_active_tokens_per_step
    assert result.request_metrics == theirs.request_metrics
    assert [(s.request_idx, s.token_ids, s.finish_reason, s.completion_step) for s in result.sequences] == [
        (s.request_idx, s.token_ids, s.finish_reason, s.completion_step) for s in theirs.sequences]
    assert result.batch_size == theirs.batch_size
    assert torch.equal(result.padded_output_tokens([2, 0]), theirs.padded_output_tokens([2, 0]))
