"""Coordinate selectors on the device (drop-in for usaf/selector.py:6-69).

``scores`` maps parameter names to CUDA tensors of importance scores.  The
global threshold is the k-th largest score over all tensors concatenated,
counting duplicates (``np.partition(arr, n-k)[n-k]`` in the reference,
usaf/selector.py:6-14), found by the radix select kernel; the masks are
``score >= threshold``, so ties are admitted and a mask may hold more than k
coordinates, exactly as in the reference.  CPU score tensors raise
``TypeError`` (there is no CPU fallback).
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

from .engine import kth_largest


def _concat(scores: Dict[str, torch.Tensor]) -> torch.Tensor:
    for name, s in scores.items():
        if not s.is_cuda:
            raise TypeError(f"usaf_b200 selectors take CUDA score tensors ({name} is on {s.device})")
    return torch.cat([s.reshape(-1).float() for s in scores.values()])


def _kth_largest_threshold(scores: Dict[str, torch.Tensor], k: int) -> float:
    """k-th largest score over all tensors, k clamped to [1, n]
    (usaf/selector.py:6-14)."""
    cat = _concat(scores)
    n = cat.numel()
    k = max(1, min(int(k), n))
    return float(kth_largest(cat, k).item())


class TopKSelector:
    """usaf/selector.py:17-26."""

    def __init__(self, k: int):
        self.k = k

    def select(self, scores: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        if not scores:
            return {}
        threshold = _kth_largest_threshold(scores, self.k)
        return {name: (s >= threshold) for name, s in scores.items()}


class ThresholdSelector:
    """usaf/selector.py:29-39: threshold = the score at ascending rank
    ``clamp(int(n * percentile / 100), 0, n-1)``."""

    def __init__(self, percentile: float):
        self.percentile = percentile

    def select(self, scores: Dict[str, torch.Tensor]) -> Dict[str, torch.Tensor]:
        cat = _concat(scores)
        n = cat.numel()
        idx = min(max(int(n * self.percentile / 100.0), 0), n - 1)
        threshold = float(kth_largest(cat, n - idx).item())   # ascending rank idx
        return {name: (s >= threshold) for name, s in scores.items()}


class DynamicSelector:
    """usaf/selector.py:42-69."""

    def __init__(self, initial_k: int, reselect_every_n_steps: int, selection: str = "topk"):
        self.initial_k = initial_k
        self.reselect_every_n_steps = reselect_every_n_steps
        self.selection = selection
        self._step_counter = 0
        self._active_mask: Dict[str, torch.Tensor] = {}

    def should_reselect(self) -> bool:
        self._step_counter += 1
        return self._step_counter % self.reselect_every_n_steps == 0

    def update_mask(self, scores: Dict[str, torch.Tensor], k: Optional[int] = None
                    ) -> Dict[str, torch.Tensor]:
        k = k or self.initial_k
        if self.selection == "topk":
            selector = TopKSelector(k)
        else:
            selector = ThresholdSelector(99.98)
        self._active_mask = selector.select(scores)
        return self._active_mask

    @property
    def active_mask(self) -> Dict[str, torch.Tensor]:
        return self._active_mask
