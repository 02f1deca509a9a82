"""One sparse training step of the MoE block, as train.py sequences it (oracle).

importance pass with ``TopKImportanceStore`` -> ``select(frac)`` (train.py:397-402)
-> fp32 masters from the original dequant (train.py:451-467) -> training pass
with ``SparseGradStore`` (train.py:408-412, 631-641) -> ``SparseAdam`` over the
masters (compact mode, train.py:490, 665) and over the full router (gather
mode; the C2 configuration trains the router with SparseAdam over all of its
coordinates).
"""
from __future__ import annotations

import numpy as np
import torch

from . import moe


PREFIX = "layer.mlp.experts"
NAMES = ("gate_up_proj", "down_proj")


def shapes_of(inp):
    E, H, I = inp["E"], inp["H"], inp["I"]
    return {f"{PREFIX}.gate_up_proj": (E, 2 * I, H), f"{PREFIX}.down_proj": (E, H, I)}


def dense_weights(inp, overlays=None):
    """Effective expert weights in the activation dtype: fp16 dequant, overlay
    values rounded to fp16 (usaf/moe_loader.py:241-247, 442), then cast to the
    activation dtype."""
    out = []
    for n in NAMES:
        full = f"{PREFIX}.{n}"
        ov = overlays.get(full) if overlays else None
        w = moe.effective_weight(inp[n]["fp16"], *(ov if ov else (None, None)))
        out.append(w.to(inp["dtype"]))
    return out


def run_step(inp, frac=0.005, lr=1e-4, experts="sparse"):
    shapes = shapes_of(inp)
    k = inp["k"]
    w_gu, w_dn = dense_weights(inp)
    imp = moe.TopKImportanceStore(shapes, frac=frac)
    moe.block_step(inp["x"], inp["w_r"], w_gu, w_dn, inp["dy"], k, True,
                   capture=imp.add, prefix=PREFIX, experts=experts)
    active = imp.select(frac)
    masters = {n: torch.from_numpy(np.ascontiguousarray(
        inp[n.rsplit(".", 1)[1]]["fp16"])).reshape(-1).index_select(0, active[n]).float()
        for n in shapes}
    overlays = {n: (active[n], masters[n]) for n in shapes}
    w_gu, w_dn = dense_weights(inp, overlays)
    store = moe.SparseGradStore(active, shapes)
    res = moe.block_step(inp["x"], inp["w_r"], w_gu, w_dn, inp["dy"], k, True,
                         capture=store.add, prefix=PREFIX, experts=experts)
    out = dict(res)
    out["active"] = active
    out["candidates"] = {n: imp.candidates(n) for n in shapes}
    out["compact"] = {n: store.compact[n].clone() for n in shapes}
    opt = moe.SparseAdam({n: masters[n].clone() for n in shapes}, active, lr=lr,
                         compact_params=True)
    opt.step(store.compact)
    out["master_after"] = {n: opt.named[n] for n in shapes}
    E, H = inp["E"], inp["H"]
    w_r = inp["w_r"].clone()
    ropt = moe.SparseAdam({"r": w_r}, {"r": torch.arange(E * H)}, lr=lr)
    ropt.step({"r": res["dW_r"]})
    out["w_r_after"] = w_r
    out["dispatch"] = moe.dispatch_indices(res["weights"])
    return out
