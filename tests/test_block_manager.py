"""Block manager behaviour the paged kernels rely on (CPU, no torch)."""

import random

import pytest

from mini_infra_b200.core import (
    NULL_BLOCK_ID, FreeKVCacheBlockQueue, KVCacheManager, Request, num_blocks_for_tokens, required_pool_blocks,
)


def test_free_queue_is_fifo_and_never_hands_out_null_block():
    q = FreeKVCacheBlockQueue(5)
    first = q.allocate(4)
    assert first == [1, 2, 3, 4] and NULL_BLOCK_ID not in first
    q.free([3, 1])
    assert q.allocate(2) == [3, 1]  # first freed, first reused
    assert q.reuse_count == 2 and q.block_cold_allocation_count == 4 and q.release_count == 2


def test_allocation_grows_only_at_block_boundaries():
    m = KVCacheManager(block_size=4, num_blocks=10)
    assert m.allocate_slots(0, 3) and m.block_table(0) == [1]
    assert m.allocate_slots(0, 1) and m.block_table(0) == [1]
    assert m.allocate_slots(0, 1) and m.block_table(0) == [1, 2]
    assert m.allocate_slots(1, 9) and m.block_table(1) == [3, 4, 5]


def test_failed_allocation_changes_nothing():
    m = KVCacheManager(block_size=2, num_blocks=4)
    assert m.allocate_slots(0, 4)
    used = m.num_used_blocks
    assert not m.allocate_slots(1, 5)
    assert m.num_used_blocks == used
    with pytest.raises(KeyError):
        m.block_table(1)


def test_admission_counts_fcfs_prefix_after_reservation():
    m = KVCacheManager(block_size=4, num_blocks=8)  # 7 free
    assert m.num_admissible([4, 8, 4, 1], num_reserved_blocks=0) == 4
    assert m.num_admissible([4, 8, 4, 1], num_reserved_blocks=3) == 3
    assert m.num_admissible([16, 1], num_reserved_blocks=4) == 0  # FCFS: head does not fit, stop


def test_required_pool_blocks_counts_longest_concurrent_requests():
    reqs = [Request(i, tuple(range(1, n + 1)), new) for i, (n, new) in enumerate([(5, 3), (17, 1), (2, 8)])]
    # peaks (prompt + new - 1): 7, 17, 9 -> blocks of 4: 2, 5, 3; two longest: 5 + 3 (+ null)
    assert required_pool_blocks(reqs, 2, 4) == 1 + 5 + 3
    assert num_blocks_for_tokens(0, 4) == 0 and num_blocks_for_tokens(9, 4) == 3


def test_free_returns_whole_table():
    m = KVCacheManager(block_size=1, num_blocks=6)
    m.allocate_slots(7, 3)
    m.free(7)
    assert m.num_used_blocks == 0 and m.block_release_count == 3


def test_live_tables_never_share_a_block_so_slots_are_unique():
    """Random admit / grow / free traffic: live block tables stay disjoint and null-free, so the
    slots of all live positions (what one step's scatter writes) have no duplicates."""
    from oracle.paged_oracle import duplicate_slots, slot_for_position

    rng = random.Random(7)
    bs = 4
    m = KVCacheManager(block_size=bs, num_blocks=40)
    lengths: dict[int, int] = {}
    for step in range(400):
        op = rng.random()
        if op < 0.4 and len(lengths) < 12:
            rid = step
            n = rng.randint(1, 20)
            if m.allocate_slots(rid, n):
                lengths[rid] = n
        elif op < 0.8 and lengths:
            rid = rng.choice(sorted(lengths))
            if m.allocate_slots(rid, 1):
                lengths[rid] += 1
        elif lengths:
            rid = rng.choice(sorted(lengths))
            m.free(rid)
            del lengths[rid]
        tables = {rid: m.block_table(rid) for rid in lengths}
        blocks = [b for t in tables.values() for b in t]
        assert NULL_BLOCK_ID not in blocks
        assert len(blocks) == len(set(blocks)) == m.num_used_blocks
        slots = [slot_for_position(tables[rid], p, bs) for rid, n in lengths.items() for p in range(n)]
        assert duplicate_slots(slots) == []


def test_duplicate_slot_detector_flags_a_planted_duplicate():
    from oracle.paged_oracle import duplicate_slots

    assert duplicate_slots([5, 9, 17, 4]) == []
    assert duplicate_slots([5, 9, 5, 4, 9, 9]) == [5, 9]
