"""Scheduler decisions (CPU): chunk planning, decode protection, admission, and step counts that
must equal what the reference engine produced on the golden C1 workloads."""

import json
from pathlib import Path

import pytest

from mini_infra_b200.core import (
    BatchingMethod, ChunkedPrefillConfig, IterationScheduler, KVCacheManager, PrefillFirstConfig, RequestState,
    SchedulePhase, SchedulerConfig, TokenBudgetConfig, make_requests, prepare_schedule,
)
from mini_infra_b200.engine import EngineConfig, validate_engine_config
from mini_infra_b200.core.types import PagedCacheConfig, DenseCacheConfig, NoCacheConfig

GOLDEN = Path(__file__).resolve().parent / "golden"


def _drive(requests, sched_cfg, block_size=16, num_blocks=None):
    """Run the scheduler with a fake backend that returns token 7 for every producer."""
    mrr = sched_cfg.max_running_requests or len(requests)
    states, arrivals, clock = prepare_schedule(requests, mrr)
    from mini_infra_b200.core.block_manager import required_pool_blocks
    nb = num_blocks or required_pool_blocks(requests, mrr, block_size)
    sch = IterationScheduler(sched_cfg.with_max_running_requests(mrr), BatchingMethod.CONTINUOUS,
                             KVCacheManager(block_size, nb))
    trace = []
    while arrivals or sch.has_unfinished_requests:
        sch.add_requests(arrivals.pop_arrived(clock))
        out = sch.schedule(clock)
        if out is None:
            clock = arrivals.next_arrival_ms()
            continue
        if out.phase is SchedulePhase.PREFILL:
            n = sum(c.is_last for c in out.prefill_chunks)
            trace.append(("P", tuple((c.start, c.end) for c in out.prefill_chunks)))
        elif out.phase is SchedulePhase.MIXED:
            n = len(out.scheduled_requests) + sum(c.is_last for c in out.prefill_chunks)
            trace.append(("M", len(out.scheduled_requests), tuple((c.start, c.end) for c in out.prefill_chunks)))
        else:
            n = len(out.scheduled_requests)
            trace.append(("D", n))
        clock += 1.0
        sch.update_from_output(out, [7] * n, clock, None, False)
    return states, trace


@pytest.mark.parametrize("case", json.loads((GOLDEN / "engine.json").read_text())["cases"], ids=lambda c: c["name"])
def test_step_counts_match_reference_engine(case):
    reqs = make_requests(case["prompts"], case["max_new_tokens"])
    policy = PrefillFirstConfig() if case["batching_policy"] == "prefill-first" else ChunkedPrefillConfig(
        case["token_budget"])
    states, trace = _drive(reqs, SchedulerConfig(case["max_running_requests"], policy))
    assert sum(t[0] == "P" for t in trace) == case["num_prefill_steps"]
    assert sum(t[0] == "D" for t in trace) == case["num_decode_steps"]
    assert all(len(s.generated) == case["max_new_tokens"] for s in states)


def test_chunked_prefill_splits_budget_and_protects_decode():
    reqs = make_requests([list(range(1, 11)), list(range(1, 4))], 3)
    _, trace = _drive(reqs, SchedulerConfig(2, ChunkedPrefillConfig(4)), block_size=2)
    # two candidates share budget 4 -> chunk cap 2; request 1 finishes its prompt first
    assert trace[0] == ("P", ((0, 2), (0, 2)))
    assert trace[1] == ("P", ((2, 4), (2, 3)))
    assert trace[2] == ("D", 1)  # decode protection after a prefill while someone decodes
    for prev, cur in zip(trace, trace[1:]):
        if prev[0] == "P" and cur[0] == "P":
            pass  # allowed only while nobody is decoding; checked by the step counts above


def test_token_budget_oversize_head_runs_alone():
    reqs = make_requests([list(range(1, 20)), [1, 2]], 1)
    _, trace = _drive(reqs, SchedulerConfig(2, TokenBudgetConfig(8)))
    assert trace[0] == ("P", ((0, 19),))


def test_engine_config_validation_rules():
    with pytest.raises(ValueError):
        validate_engine_config(EngineConfig(PagedCacheConfig(16), BatchingMethod.NONE))
    with pytest.raises(ValueError):
        validate_engine_config(EngineConfig(DenseCacheConfig(), BatchingMethod.CONTINUOUS,
                                            scheduler_config=SchedulerConfig(None, ChunkedPrefillConfig(8))))
    with pytest.raises(ValueError):
        validate_engine_config(EngineConfig(PagedCacheConfig(16), BatchingMethod.CONTINUOUS,
                                            scheduler_config=SchedulerConfig(16, ChunkedPrefillConfig(8))))
    with pytest.raises(ValueError):
        validate_engine_config(EngineConfig(NoCacheConfig(), BatchingMethod.CONTINUOUS))
    validate_engine_config(EngineConfig(PagedCacheConfig(16), BatchingMethod.CONTINUOUS,
                                        scheduler_config=SchedulerConfig(8, ChunkedPrefillConfig(64))))


def test_exhausted_pool_fails_loudly():
    reqs = make_requests([list(range(1, 9)), list(range(1, 9))], 8)
    with pytest.raises(RuntimeError):
        _drive(reqs, SchedulerConfig(2, PrefillFirstConfig()), block_size=4, num_blocks=5)


def test_mixed_chunked_prefill_packs_decode_rows_and_budgeted_chunks():
    """ChunkedPrefillConfig(mixed=True): once a request decodes, each step carries every decode
    row plus chunks planned from the remaining budget (token_budget - decode rows)."""
    reqs = make_requests([list(range(1, 4)), list(range(1, 11))], 4)
    budget = 6
    states, trace = _drive(reqs, SchedulerConfig(2, ChunkedPrefillConfig(budget, mixed=True)), block_size=2)
    assert trace[0] == ("P", ((0, 3), (0, 3)))          # nothing decodes yet: a plain prefill, cap 6 // 2
    assert trace[1] == ("M", 1, ((3, 8),))               # 1 decode row + a chunk of 6 - 1 = 5 tokens
    assert trace[2] == ("M", 1, ((8, 10),))              # the last chunk rides with the next decode token
    assert all(t[0] == "D" for t in trace[3:])           # both decode: nothing left to prefill
    for t in trace:
        if t[0] == "M":
            assert sum(e - b for b, e in t[2]) <= budget - t[1] and len(t[2]) <= budget - t[1]
    assert all(len(s.generated) == 4 for s in states)


def test_mixed_flag_is_off_by_default_and_named():
    assert ChunkedPrefillConfig(8).mixed is False
    assert str(ChunkedPrefillConfig(8, mixed=True)) == "chunked-prefill(token_budget=8, mixed)"
