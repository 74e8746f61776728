"""Stateless model runner base (reference ``worker/base_runner.py``): holds the model, its device
and the pad token; ``run_prefill_step`` prefills whole prompts (left padding, no history)."""

from __future__ import annotations

from collections.abc import Sequence
from typing import NamedTuple

import torch

from mini_infra_b200.worker.kv_cache import KVCache


class PrefillOutput(NamedTuple):
    next_tokens: list[int]
    prefill_cache: KVCache
    model_ms: float


def _left_pad_sequences(
    token_sequences: Sequence[Sequence[int]], pad_token_id: int, device: torch.device
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """[B, L] input ids (left-padded), bool mask, positions (0 on padding) and prompt lengths."""
    if not token_sequences:
        raise ValueError("token_sequences must not be empty")
    lens = [len(s) for s in token_sequences]
    if min(lens) < 1:
        raise ValueError("every prompt must be a non-empty 1-D token sequence")
    width = max(lens)
    ids = [[pad_token_id] * (width - n) + [int(t) for t in s] for s, n in zip(token_sequences, lens)]
    input_ids = torch.tensor(ids, dtype=torch.long, device=device)
    mask = torch.arange(width, device=device).unsqueeze(0) >= torch.tensor(
        [width - n for n in lens], device=device).unsqueeze(1)
    positions = (mask.long().cumsum(dim=-1) - 1).clamp_(min=0)
    return input_ids, mask, positions, torch.tensor(lens, dtype=torch.long, device=device)


class BaseModelRunner:
    def __init__(self, model: torch.nn.Module, pad_token_id: int = 0):
        self.model = model
        self.device = next(model.parameters()).device
        self.pad_token_id = pad_token_id

    def run_prefill_step(self, prompt_sequences: Sequence[Sequence[int]]) -> PrefillOutput:
        """Whole-prompt prefill of new requests: a chunk step whose rows all start at position 0."""
        return self.run_prefill_chunk_step(  # type: ignore[attr-defined]
            prompt_sequences, [0] * len(prompt_sequences), [[] for _ in prompt_sequences], None
        )


__all__ = ["BaseModelRunner", "PrefillOutput"]
