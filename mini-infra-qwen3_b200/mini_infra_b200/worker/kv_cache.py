"""Per-layer K/V handed from a prefill forward to ``PagedRunner.store_prefill``.

``PrefillOutput.prefill_cache`` is one of these (the reference's ``worker/kv_cache.py`` container,
whose attribute names callers use).  Each layer holds its chunk's keys and values as
``[batch, num_kv_heads, length, head_dim]`` tensors — here transposed views of the model's
``[batch, length, heads, head_dim]`` projections, so building the cache copies nothing; valid tokens
are right-aligned in ``length`` (left padding).
"""

from __future__ import annotations

from collections.abc import Sequence

import torch


class KVCache:
    """Layer-indexed (key, value) pairs; ``key_cache`` / ``value_cache`` are the per-layer lists."""

    def __init__(self, past_key_values: Sequence[tuple[torch.Tensor, torch.Tensor]] | None = None):
        layers = () if past_key_values is None else past_key_values
        self.key_cache: list[torch.Tensor] = [k for k, _ in layers]
        self.value_cache: list[torch.Tensor] = [v for _, v in layers]

    @property
    def past_key_values(self) -> list[tuple[torch.Tensor, torch.Tensor]]:
        """The layers as (key, value) pairs, the form the model's forward returns them in."""
        return list(zip(self.key_cache, self.value_cache))

    @property
    def length(self) -> int:
        """Padded token length of the chunk (0 for an empty cache)."""
        return self.key_cache[0].shape[2] if self.key_cache else 0

    @property
    def total_bytes(self) -> int:
        """Bytes the layers' tensors span (views count their own extent, not their base's)."""
        return sum(k.numel() * k.element_size() + v.numel() * v.element_size()
                   for k, v in zip(self.key_cache, self.value_cache))

    def __len__(self) -> int:
        return len(self.key_cache)

    def __iter__(self):
        return iter(zip(self.key_cache, self.value_cache))

    def __getitem__(self, layer_idx: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.key_cache[layer_idx], self.value_cache[layer_idx]


def cache_size_bytes(kv_cache) -> int:
    """Bytes of a KVCache or of a plain sequence of (key, value) pairs; 0 for None."""
    if kv_cache is None:
        return 0
    if isinstance(kv_cache, KVCache):
        return kv_cache.total_bytes
    return sum(k.numel() * k.element_size() + v.numel() * v.element_size() for k, v in kv_cache)
