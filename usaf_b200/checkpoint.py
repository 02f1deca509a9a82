"""Sparse checkpoints of device training state (drop-in for usaf/checkpoint.py).

The file format is the reference's ``usaf-sparse-v1`` (usaf/checkpoint.py:20-47):
a ``torch.save`` dict with the active indices, the fp32 masters and the
optimizer state, all as CPU tensors, so files written here load in the
reference and the other way round.  Saving copies the device state to the
host; loading returns CPU tensors (the caller moves them to its device, as
``SparseMoELayer.init_selection_from`` does).

``export_merged_weights`` (usaf/checkpoint.py:58-92) merges the trained
coordinates into the original int4 weights -- dequantize, scatter
``fp16(master)``, re-quantize -- with the int4 kernels on the device.  Both
kernels are bit-exact with the reference, so the exported file equals the
reference's export of the same inputs.
"""
from __future__ import annotations

import os
import time
from typing import Any, Dict, List, Optional

import torch

from .quantization import dequantize_4bit, quantize_state_dict


def save_sparse_checkpoint(path: str, masters: Dict[str, torch.Tensor],
                           active_idx: Dict[str, torch.Tensor], optimizer_state: Dict[str, Any],
                           config: Dict[str, Any], step: int, losses: List[float],
                           train_layers: List[int], metric: Optional[float] = None) -> str:
    """usaf/checkpoint.py:20-47."""
    path = str(path)
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    state = {
        "format": "usaf-sparse-v1",
        "timestamp": time.time(),
        "step": step,
        "losses": losses,
        "train_layers": train_layers,
        "config": config,
        "metric": metric,
        "active_idx": {k: v.detach().cpu() for k, v in active_idx.items()},
        "masters": {k: v.detach().cpu() for k, v in masters.items()},
        "optimizer": _to_cpu(optimizer_state),
    }
    torch.save(state, path)
    return path


def _to_cpu(obj):
    if isinstance(obj, torch.Tensor):
        return obj.detach().cpu()
    if isinstance(obj, dict):
        return {k: _to_cpu(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return type(obj)(_to_cpu(v) for v in obj)
    return obj


def load_sparse_checkpoint(path: str) -> Dict[str, Any]:
    """usaf/checkpoint.py:50-55: ``ValueError`` unless the file is usaf-sparse-v1."""
    state = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(state, dict) or state.get("format") != "usaf-sparse-v1":
        raise ValueError(f"Not a valid USAF sparse checkpoint: {path}")
    return state


def get_checkpoint_metadata(path: str) -> Dict[str, Any]:
    """usaf/checkpoint.py:95-110."""
    state = torch.load(path, map_location="cpu", weights_only=True)
    if not isinstance(state, dict):
        return {"error": "invalid checkpoint"}
    return {
        "format": state.get("format", "unknown"),
        "step": state.get("step", -1),
        "losses": state.get("losses", []),
        "n_active": sum(v.numel() for v in state.get("active_idx", {}).values()),
        "n_masters": len(state.get("masters", {})),
        "train_layers": state.get("train_layers", []),
        "timestamp": state.get("timestamp", 0),
        "config": state.get("config", {}),
        "metric": state.get("metric"),
    }


def export_merged_weights(quant_path: str, masters: Dict[str, torch.Tensor],
                          active_idx: Dict[str, torch.Tensor], output_path: str,
                          group_size: int = 128, device=None) -> str:
    """usaf/checkpoint.py:58-92 on the device: every q4 entry is dequantized to
    fp16, the trained coordinates are replaced by ``fp16(master)``, and the
    merged tensors are re-quantized (``quantize_state_dict``); the result is
    written with CPU tensors."""
    dev = torch.device(device) if device is not None else torch.device("cuda")
    q_dict: Dict[str, Any] = torch.load(quant_path, map_location="cpu", weights_only=True)
    merged: Dict[str, torch.Tensor] = {}
    for fname, entry in q_dict.items():
        if isinstance(entry, dict) and "q" in entry:
            t = dequantize_4bit(entry["q"].to(dev), entry["s"].to(dev), entry["z"].to(dev),
                                entry["shape"], group_size=entry.get("group_size", group_size))
        elif isinstance(entry, torch.Tensor):
            t = entry.to(device=dev, dtype=torch.float16)
        else:
            continue
        if fname in masters and fname in active_idx:
            aidx = active_idx[fname].reshape(-1).to(device=dev, dtype=torch.long)
            trained = masters[fname].detach().to(device=dev, dtype=torch.float16).reshape(-1)
            if aidx.numel() != trained.numel():
                raise ValueError(f"{fname}: {trained.numel()} masters for {aidx.numel()} indices")
            if aidx.numel() and (int(aidx.min()) < 0 or int(aidx.max()) >= t.numel()):
                raise IndexError(f"{fname}: active index out of range")
            flat = t.reshape(-1).clone()
            flat.scatter_(0, aidx, trained)
            t = flat.reshape(t.shape)
        merged[fname] = t
    merged_q4 = _to_cpu(quantize_state_dict(merged, group_size=group_size))
    torch.save(merged_q4, output_path)
    return output_path
