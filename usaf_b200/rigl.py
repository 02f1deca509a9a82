"""RigL reselection merge on the device (train.py:536-613).

Per tensor: ``kept = sorted(old & new)``, ``grown = sorted(new - old)[:len(old) -
len(kept)]``, ``final = kept + grown`` (train.py:559-565).  Kept coordinates
carry their trained master (:575-583); grown ones restart from the ORIGINAL
int4 dequant (:585-593).  The caller then builds a fresh SparseAdam, so m, v
and the step count reset (:610).  Sorting uses the library's stable radix
sort; membership is a binary search into the sorted old list.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import engine


def merge(old: torch.Tensor, new: Optional[torch.Tensor], old_masters: torch.Tensor,
          original_flat: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    dev = old.device
    n_old = old.numel()
    if new is None or new.numel() == 0 or n_old == 0:
        # nothing new, or nothing to replace: the budget is len(old) (train.py:563-565)
        return old.clone(), old_masters.clone()
    old_s, old_pos = engine.sort_u32(old, torch.arange(n_old, device=dev))
    new_s, _ = engine.sort_u32(new.to(dev), torch.arange(new.numel(), device=dev))
    old_s = old_s.long()
    new_s = new_s.long()
    loc = torch.searchsorted(old_s, new_s).clamp_max(n_old - 1)
    in_old = old_s[loc] == new_s
    kept = new_s[in_old]
    cand = new_s[~in_old]
    fill = max(0, n_old - kept.numel())
    grown = cand[:fill]
    final = torch.cat([kept, grown])
    vals = torch.empty(final.numel(), dtype=torch.float32, device=dev)
    nk = kept.numel()
    if nk:
        vals[:nk] = old_masters.float()[old_pos[loc[in_old]]]
    if grown.numel():
        vals[nk:] = original_flat.reshape(-1)[grown].float()
    return final, vals
