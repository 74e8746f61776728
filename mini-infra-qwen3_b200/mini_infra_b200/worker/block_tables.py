"""Device mirror of the live block tables, one row per batch slot.

The reference rebuilds every decode step's block tables on the host, null-padded to the longest
(``worker/paged_runner.py:152-162``): O(batch x max_blocks) Python integers per step, ~1 M at a
batch of 512 with 32 K-token contexts.  Here each batch slot owns one row of a device tensor
``[capacity, width]`` that holds the block table of the sequence in that slot; a step sends only
the entries added since the slot's last step (a sequence gains one block every block_size
tokens) together with (slot, token, position) per sequence, and ``mi_decode_rows`` builds the
step's packed inputs on the device.

A slot's row is identified with its sequence by a key (the request id): a new key in a slot
resends that sequence's whole table once.  Tables only grow while their sequence holds its slot
(the block manager appends and frees whole tables; there is no preemption), which is what makes
"entries past the last synced length" the complete change.  As a guard against a caller that
rebuilds a table under the same key, a slot whose table is shorter than what was synced, or whose
last synced entry changed, is resent whole.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch


class DeviceBlockTables:
    def __init__(self, capacity: int, width: int, device: torch.device):
        if capacity < 1 or width < 1:
            raise ValueError(f"capacity and width must be positive (got {capacity}, {width})")
        self.capacity = capacity
        self.width = width
        self.tables = torch.zeros((capacity, width), dtype=torch.long, device=device)
        self._owner = [None] * capacity  # key of the sequence whose table the row holds
        self._synced = [0] * capacity  # entries of that table already on the device
        self._last = [0] * capacity  # the last of those entries (block id)

    def step_inputs(
        self,
        row_keys: Sequence[tuple[int, int]],
        block_tables: Sequence[Sequence[int]],
        last_tokens: Sequence[int],
        positions: Sequence[int],
    ) -> tuple[np.ndarray, int, int]:
        """One int64 host array: rows [B, 3] (slot, token, position) then the table entries to
        write [D, 3] (slot, column, block id); returns (array, B, D) and records the entries as
        synced."""
        rows: list[int] = []
        deltas: list[int] = []
        for (slot, key), table, token, pos in zip(row_keys, block_tables, last_tokens, positions):
            if not 0 <= slot < self.capacity:
                raise ValueError(f"batch slot {slot} outside [0, {self.capacity})")
            if len(table) > self.width:
                raise ValueError(f"a block table of {len(table)} blocks exceeds the device tables' width {self.width}")
            start = self._synced[slot]
            if self._owner[slot] != key or len(table) < start or (start and int(table[start - 1]) != self._last[slot]):
                self._owner[slot] = key
                start = 0
            for col in range(start, len(table)):
                deltas += (slot, col, int(table[col]))
            self._synced[slot] = len(table)
            if len(table):
                self._last[slot] = int(table[-1])
            rows += (slot, int(token), int(pos))
        return np.asarray(rows + deltas, dtype=np.int64), len(rows) // 3, len(deltas) // 3


__all__ = ["DeviceBlockTables"]
