"""Device synchronisation, per-step timing and memory statistics (reference ``device.py`` API)."""

from __future__ import annotations

import time
from types import TracebackType

import torch


def synchronize(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.synchronize(device)


class StepTimer:
    """Times one step: synchronize, CUDA event, work, CUDA event, synchronize (wall clock off CUDA)."""

    def __init__(self, device: torch.device):
        self.device = device
        self.elapsed_ms = 0.0
        self._events: tuple[torch.cuda.Event, torch.cuda.Event] | None = None
        self._t0 = 0.0

    def __enter__(self) -> "StepTimer":
        if self.device.type == "cuda":
            synchronize(self.device)
            self._events = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self._events[0].record()
        else:
            self._t0 = time.perf_counter()
        return self

    def __exit__(self, exc_type: type[BaseException] | None, exc: BaseException | None, tb: TracebackType | None):
        if self._events is not None:
            self._events[1].record()
            synchronize(self.device)
            self.elapsed_ms = self._events[0].elapsed_time(self._events[1])
        else:
            self.elapsed_ms = (time.perf_counter() - self._t0) * 1000.0


def reset_peak_memory(device: torch.device) -> None:
    if device.type == "cuda":
        torch.cuda.reset_peak_memory_stats(device)


def allocated_memory_mb(device: torch.device) -> float:
    return torch.cuda.memory_allocated(device) / 2**20 if device.type == "cuda" else 0.0


def peak_memory_mb(device: torch.device) -> tuple[float, float]:
    if device.type != "cuda":
        return 0.0, 0.0
    return torch.cuda.max_memory_allocated(device) / 2**20, torch.cuda.max_memory_reserved(device) / 2**20
