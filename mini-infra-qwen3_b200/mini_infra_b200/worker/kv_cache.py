"""Explicit per-layer K/V container (reference ``worker/kv_cache.py``): tensors [B, H_kv, L, D]."""

from __future__ import annotations

from collections.abc import Sequence

import torch


class KVCache:
    def __init__(self, past_key_values: Sequence[tuple[torch.Tensor, torch.Tensor]] | None = None):
        layers = () if past_key_values is None else past_key_values
        self.key_cache: list[torch.Tensor] = [k for k, _ in layers]
        self.value_cache: list[torch.Tensor] = [v for _, v in layers]

    @property
    def past_key_values(self) -> list[tuple[torch.Tensor, torch.Tensor]]:
        return list(zip(self.key_cache, self.value_cache))

    @property
    def length(self) -> int:
        return self.key_cache[0].shape[2] if self.key_cache else 0

    @property
    def total_bytes(self) -> int:
        return sum(k.numel() * k.element_size() + v.numel() * v.element_size()
                   for k, v in zip(self.key_cache, self.value_cache))

    def __len__(self) -> int:
        return len(self.key_cache)

    def __iter__(self):
        return iter(zip(self.key_cache, self.value_cache))

    def __getitem__(self, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.key_cache[layer_idx], self.value_cache[layer_idx]


def cache_size_bytes(kv_cache) -> int:
    if kv_cache is None:
        return 0
    if isinstance(kv_cache, KVCache):
        return kv_cache.total_bytes
    return sum(k.numel() * k.element_size() + v.numel() * v.element_size() for k, v in kv_cache)
