"""Logical block allocation of the paged KV cache (pure Python: the control plane never imports torch).

Behaviour kept from the reference's ``core/block_manager.py``, because its tests and every kernel
input depend on it:

* block ``NULL_BLOCK_ID`` (0) is never handed out; it right-pads block tables;
* free blocks are handed out in the order they became free, the never-used ones first (FIFO);
* a request's table grows only when its cached token count crosses a block boundary, and an
  allocation that does not fit changes nothing and returns False;
* admission takes the longest first-come-first-served prefix of waiting prompts whose blocks fit
  after the blocks still owed to in-flight chunked prefills;
* the counters ``block_cold_allocation_count`` (first hand-out of a block id), ``block_reuse_count``,
  ``block_release_count`` and ``peak_used_blocks``.

Design here: the free list is a fixed-capacity ring over the num_blocks - 1 allocatable ids (a
block id is either in the ring or in exactly one table, so the ring never overflows); a bytearray
marks the ids handed out before; each request holds a lease of its table and cached token count;
admission is a bisection over the prefix sums of the waiting prompts' block needs.
"""

from __future__ import annotations

import bisect
import heapq
import itertools
from collections.abc import Iterable, Sequence
from dataclasses import dataclass, field

from mini_infra_b200.core.request import Request

NULL_BLOCK_ID = 0


def num_blocks_for_tokens(num_tokens: int, block_size: int) -> int:
    """Blocks needed to hold num_tokens tokens (ceiling division)."""
    return -(-num_tokens // block_size)


def required_pool_blocks(requests: Sequence[Request], max_running_requests: int | None, block_size: int) -> int:
    """Pool size, the null block included, that no max_running_requests concurrent requests can
    exhaust: the blocks of the largest peaks.  A request's peak is prompt_len + max_new_tokens - 1
    cached tokens (its last generated token is never fed back, so its K/V are never written)."""
    peaks = (r.prompt_len + r.max_new_tokens - 1 for r in requests)
    limit = len(requests) if max_running_requests is None else max_running_requests
    return 1 + sum(num_blocks_for_tokens(p, block_size) for p in heapq.nlargest(limit, peaks))


class FreeKVCacheBlockQueue:
    """FIFO of the free physical block ids 1 .. num_blocks - 1, with allocation counters."""

    def __init__(self, num_blocks: int):
        if num_blocks < 2:
            raise ValueError(f"num_blocks must be at least 2, block {NULL_BLOCK_ID} being the null block "
                             f"(got {num_blocks})")
        self.num_blocks = num_blocks
        self._ring = list(range(NULL_BLOCK_ID + 1, num_blocks))
        self._head = 0  # ring index of the next block handed out
        self._free = len(self._ring)  # free ids at ring[head], ring[head + 1], ... (cyclically)
        self._handed_out_before = bytearray(num_blocks)
        self.block_cold_allocation_count = 0
        self.reuse_count = 0
        self.release_count = 0
        self.peak_used_blocks = 0

    @property
    def num_free_blocks(self) -> int:
        return self._free

    @property
    def num_used_blocks(self) -> int:
        return len(self._ring) - self._free

    def allocate(self, num_blocks: int) -> list[int]:
        """The next num_blocks free ids, oldest-freed first; RuntimeError if fewer are free."""
        if num_blocks > self._free:
            raise RuntimeError(f"out of free blocks (空闲块不足): {num_blocks} requested, {self._free} free")
        cap = len(self._ring)
        taken = [self._ring[(self._head + i) % cap] for i in range(num_blocks)]
        self._head = (self._head + num_blocks) % cap
        self._free -= num_blocks
        cold = sum(1 for b in taken if not self._handed_out_before[b])
        for b in taken:
            self._handed_out_before[b] = 1
        self.block_cold_allocation_count += cold
        self.reuse_count += num_blocks - cold
        self.peak_used_blocks = max(self.peak_used_blocks, self.num_used_blocks)
        return taken

    def free(self, block_ids: Iterable[int]) -> None:
        """Return ids to the back of the queue, in the order given."""
        cap = len(self._ring)
        released = 0
        for b in block_ids:
            if not NULL_BLOCK_ID < b < self.num_blocks:
                raise ValueError(f"block id {b} is not an allocatable block of this pool")
            if self._free == cap:
                raise RuntimeError("more blocks freed than were handed out")
            self._ring[(self._head + self._free) % cap] = b
            self._free += 1
            released += 1
        self.release_count += released


@dataclass
class _Lease:
    """One request's physical blocks (logical block i -> table[i]) and its cached token count."""

    table: list[int] = field(default_factory=list)
    tokens: int = 0


class KVCacheManager:
    """Per-request block tables over one FreeKVCacheBlockQueue, grown on demand."""

    def __init__(self, block_size: int, num_blocks: int):
        if block_size < 1:
            raise ValueError(f"block_size must be positive (got {block_size})")
        self.block_size = block_size
        self.free_block_queue = FreeKVCacheBlockQueue(num_blocks)
        self._leases: dict[int, _Lease] = {}

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
        """The request's table (KeyError for a request holding no lease)."""
        return self._leases[request_idx].table

    def num_admissible(self, prompt_lens: Sequence[int], num_reserved_blocks: int) -> int:
        """How many of the waiting prompts, taken in order, fit in the free blocks left after
        num_reserved_blocks (a prompt that does not fit stops admission: no overtaking)."""
        budget = self.free_block_queue.num_free_blocks - num_reserved_blocks
        needs = (num_blocks_for_tokens(n, self.block_size) for n in prompt_lens)
        return bisect.bisect_right(list(itertools.accumulate(needs)), budget)

    def allocate_slots(self, request_idx: int, num_new_tokens: int) -> bool:
        """Make room for num_new_tokens more cached tokens of the request; False (and no change)
        when the blocks that takes are not free."""
        lease = self._leases.get(request_idx)
        held = len(lease.table) if lease is not None else 0
        tokens = (lease.tokens if lease is not None else 0) + num_new_tokens
        missing = num_blocks_for_tokens(tokens, self.block_size) - held
        if missing > self.free_block_queue.num_free_blocks:
            return False
        if lease is None:
            lease = self._leases[request_idx] = _Lease()
        lease.table += self.free_block_queue.allocate(max(missing, 0))
        lease.tokens = tokens
        return True

    def free(self, request_idx: int) -> None:
        """Release the request's blocks (KeyError for a request holding no lease)."""
        self.free_block_queue.free(self._leases.pop(request_idx).table)


__all__ = ["FreeKVCacheBlockQueue", "KVCacheManager", "NULL_BLOCK_ID", "num_blocks_for_tokens", "required_pool_blocks"]
