"""Per-layer physical block pools of the paged KV cache (reference ``worker/paged_kv_cache.py``).

Same contract: each layer holds (key_pool, value_pool), each [num_blocks, block_size, H_kv, D],
zero-initialised (freed blocks are not cleared; readers mask by context length, and zeros keep
every stale value finite); block 0 is the null block; slot = block * block_size + offset on the
flattened [num_blocks * block_size, H_kv, D] view.  The copies run on the CUDA kernels of
``libmi_paged.so`` (one launch moves K and V of one layer).  With head partitioning each process
holds only its KV heads.
"""

from __future__ import annotations

import math

import torch

from mini_infra_b200 import ops
from mini_infra_b200.worker.kv_cache import KVCache


class PagedKVCachePool:
    def __init__(
        self,
        num_layers: int,
        num_blocks: int,
        block_size: int,
        num_kv_heads: int,
        head_dim: int,
        dtype: torch.dtype,
        device: torch.device,
    ):
        if torch.device(device).type != "cuda":
            raise RuntimeError("PagedKVCachePool lives in GPU memory; this package has no CPU path")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        shape = (num_blocks, block_size, num_kv_heads, head_dim)
        self.kv_pools: list[tuple[torch.Tensor, torch.Tensor]] = [
            (torch.zeros(shape, dtype=dtype, device=device), torch.zeros(shape, dtype=dtype, device=device))
            for _ in range(num_layers)
        ]

    @property
    def bytes_per_block(self) -> int:
        """K+V bytes of one block across all layers."""
        key_pool = self.kv_pools[0][0]
        return 2 * len(self.kv_pools) * math.prod(key_pool.shape[1:]) * key_pool.element_size()

    @property
    def total_bytes(self) -> int:
        return self.num_blocks * self.bytes_per_block

    def gather_blocks(self, block_ids: torch.Tensor) -> tuple[tuple[torch.Tensor, torch.Tensor], ...]:
        """Per layer (key, value) history [B, H_kv, nb * bs, D] (transposed views of block copies)."""
        b, nb = block_ids.shape
        shape = (b, nb * self.block_size, self.num_kv_heads, self.head_dim)
        return tuple(
            (ops.gather_blocks(kp, block_ids).view(shape).transpose(1, 2),
             ops.gather_blocks(vp, block_ids).view(shape).transpose(1, 2))
            for kp, vp in self.kv_pools
        )

    def write_prefill(
        self,
        prefill_cache: KVCache,
        token_rows: torch.Tensor,
        token_positions: torch.Tensor,
        slot_mapping: torch.Tensor,
    ) -> None:
        """Scatter every valid token of every layer: pool slot_mapping[i] <- (token_rows[i], :, token_positions[i], :)."""
        for (kp, vp), (key, value) in zip(self.kv_pools, prefill_cache):
            ops.kv_scatter(key, value, token_rows, token_positions, slot_mapping, kp, vp)

    def store_chunks(
        self,
        prefill_cache: KVCache,
        chunk_lens: torch.Tensor,
        start_positions: torch.Tensor,
        block_tables: torch.Tensor,
    ) -> None:
        """Scatter right-aligned chunks with the slots computed on the device from the block tables."""
        for (kp, vp), (key, value) in zip(self.kv_pools, prefill_cache):
            ops.kv_store_chunks(key, value, chunk_lens, start_positions, block_tables, kp, vp)


__all__ = ["PagedKVCachePool"]
