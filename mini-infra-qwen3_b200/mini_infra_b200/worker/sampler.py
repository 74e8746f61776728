"""Greedy sampling of the last position (reference ``worker/sampler.py``)."""

import torch


def greedy_sample(logits: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """logits [B, L, V] -> (next_token [B, 1] int64, last_logits [B, V])."""
    last = logits[:, -1, :]
    return torch.argmax(last, dim=-1, keepdim=True), last
