"""Logical block allocation for the paged KV cache (no torch).

Same contract as the reference's ``core/block_manager.py``:

* block 0 is the null block: never handed out, used to right-pad block tables (:16-17);
* free blocks are reused first-freed-first (FIFO), which the reference's tests pin (:35-76);
* a request's block table grows only when its token count crosses a block boundary, and an
  allocation that does not fit changes nothing and reports False (:134-144);
* admission counts, FCFS, how many waiting prompts fit after reserving the blocks still owed to
  in-flight chunked prefills (:118-132).
"""

from __future__ import annotations

from collections import deque
from collections.abc import Sequence

from mini_infra_b200.core.request import Request
from mini_infra_b200.core.types import PagedCacheConfig

NULL_BLOCK_ID = 0


def num_blocks_for_tokens(num_tokens: int, block_size: int) -> int:
    return -(-num_tokens // block_size)


def required_pool_blocks(requests: Sequence[Request], max_running_requests: int, block_size: int) -> int:
    """Pool size (incl. the null block) that no set of max_running_requests concurrent requests
    can exhaust.  A request caches at most prompt_len + max_new_tokens - 1 tokens: its last
    generated token is never fed back, so its K/V are never written."""
    peaks = sorted((r.prompt_len + r.max_new_tokens - 1 for r in requests), reverse=True)
    return 1 + sum(num_blocks_for_tokens(n, block_size) for n in peaks[:max_running_requests])


class FreeKVCacheBlockQueue:
    """FIFO of free physical block ids (1 .. num_blocks-1) with reuse counters."""

    def __init__(self, num_blocks: int):
        if num_blocks < 2:
            raise ValueError("num_blocks must be >= 2 (block 0 is the null block)")
        self.num_blocks = num_blocks
        self._free: deque[int] = deque(range(NULL_BLOCK_ID + 1, num_blocks))
        self._seen: set[int] = set()
        self.block_cold_allocation_count = 0
        self.reuse_count = 0
        self.release_count = 0
        self.peak_used_blocks = 0

    @property
    def num_free_blocks(self) -> int:
        return len(self._free)

    @property
    def num_used_blocks(self) -> int:
        return self.num_blocks - 1 - len(self._free)

    def allocate(self, num_blocks: int) -> list[int]:
        if num_blocks > len(self._free):
            raise RuntimeError(f"out of free blocks: need {num_blocks}, have {len(self._free)}")
        out = [self._free.popleft() for _ in range(num_blocks)]
        for block in out:
            if block in self._seen:
                self.reuse_count += 1
            else:
                self._seen.add(block)
                self.block_cold_allocation_count += 1
        self.peak_used_blocks = max(self.peak_used_blocks, self.num_used_blocks)
        return out

    def free(self, block_ids: Sequence[int]) -> None:
        self._free.extend(block_ids)
        self.release_count += len(block_ids)


class KVCacheManager:
    """Per-request block tables (logical block i -> physical block id), grown on demand."""

    def __init__(self, block_size: int, num_blocks: int):
        if block_size < 1:
            raise ValueError("block_size must be positive")
        self.block_size = block_size
        self.free_block_queue = FreeKVCacheBlockQueue(num_blocks)
        self._tables: dict[int, list[int]] = {}
        self._tokens: dict[int, int] = {}

    @property
    def num_used_blocks(self) -> int:
        return self.free_block_queue.num_used_blocks

    @property
    def block_cold_allocation_count(self) -> int:
        return self.free_block_queue.block_cold_allocation_count

    @property
    def block_reuse_count(self) -> int:
        return self.free_block_queue.reuse_count

    @property
    def block_release_count(self) -> int:
        return self.free_block_queue.release_count

    @property
    def peak_used_blocks(self) -> int:
        return self.free_block_queue.peak_used_blocks

    def block_table(self, request_idx: int) -> list[int]:
        return self._tables[request_idx]

    def num_admissible(self, prompt_lens: Sequence[int], num_reserved_blocks: int) -> int:
        budget = self.free_block_queue.num_free_blocks - num_reserved_blocks
        count = 0
        for n in prompt_lens:
            need = num_blocks_for_tokens(n, self.block_size)
            if need > budget:
                break
            budget -= need
            count += 1
        return count

    def allocate_slots(self, request_idx: int, num_new_tokens: int) -> bool:
        table = self._tables.get(request_idx, [])
        total = self._tokens.get(request_idx, 0) + num_new_tokens
        extra = num_blocks_for_tokens(total, self.block_size) - len(table)
        if extra > self.free_block_queue.num_free_blocks:
            return False
        table.extend(self.free_block_queue.allocate(extra))
        self._tables[request_idx] = table
        self._tokens[request_idx] = total
        return True

    def free(self, request_idx: int) -> None:
        self.free_block_queue.free(self._tables.pop(request_idx))
        del self._tokens[request_idx]


__all__ = [
    "FreeKVCacheBlockQueue",
    "KVCacheManager",
    "NULL_BLOCK_ID",
    "PagedCacheConfig",
    "num_blocks_for_tokens",
    "required_pool_blocks",
]
