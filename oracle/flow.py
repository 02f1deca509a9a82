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


def masters_of(inp, active):
    """fp32 masters from the original int4 dequant (fp16) at the active
    coordinates (train.py:451-467)."""
    return {n: torch.from_numpy(np.ascontiguousarray(inp[n.rsplit(".", 1)[1]]["fp16"]))
            .reshape(-1).index_select(0, active[n].reshape(-1).long()).float() for n in active}


def step_dys(inp, steps):
    """The upstream gradient of each step of a trajectory: step s uses dY
    rolled by s tokens, so every step sees a different gradient."""
    return [torch.roll(inp["dy"], s, 0).contiguous() for s in range(steps)]


def run_trajectory(inp, active, steps=3, lr=1e-4, router_lr=None, router="adam",
                   weight_decay=0.01, experts="sparse", write_back=True):
    """``steps`` training steps on a fixed active set (train.py:630-672 per
    step, accum 1, loss scale 1).

    Each step builds the effective expert weights from the CURRENT masters
    (``_get_resident`` after ``sync_resident``, usaf/moe_loader.py:226-247,
    425-443), runs forward + backward with ``SparseGradStore`` capture, then
    steps SparseAdam over the compact masters (usaf/sparse_optim.py:86-134)
    and the router: ``router="adam"`` is SparseAdam over all of W_r (gather
    mode), ``router="sgd"`` is train.py's SGD with momentum 0.9 and weight
    decay (train.py:494-498, 667-672).  ``write_back=False`` freezes the
    overlays at the initial masters (a planted fault: what a lost
    ``sync_resident`` would compute).  Returns one dict per step."""
    shapes = shapes_of(inp)
    k = inp["k"]
    E, H = inp["E"], inp["H"]
    router_lr = lr if router_lr is None else router_lr
    masters = masters_of(inp, active)
    frozen = {n: m.clone() for n, m in masters.items()}
    opt = moe.SparseAdam(masters, active, lr=lr, weight_decay=weight_decay,
                         compact_params=True)
    w_r = inp["w_r"].clone()
    if router == "adam":
        ropt = moe.SparseAdam({"r": w_r}, {"r": torch.arange(E * H)}, lr=router_lr,
                              weight_decay=weight_decay)
        rparam = None
    elif router == "sgd":
        rparam = torch.nn.Parameter(w_r, requires_grad=False)
        ropt = torch.optim.SGD([rparam], lr=router_lr, momentum=0.9, weight_decay=weight_decay)
    else:
        raise ValueError(router)
    out = []
    for dy in step_dys(inp, steps):
        ov = masters if write_back else frozen
        w_gu, w_dn = dense_weights(inp, {n: (active[n], ov[n]) for n in shapes})
        store = moe.SparseGradStore(active, shapes)
        res = moe.block_step(inp["x"], w_r, w_gu, w_dn, dy, k, True, capture=store.add,
                             prefix=PREFIX, experts=experts)
        opt.step(store.compact)
        if router == "adam":
            ropt.step({"r": res["dW_r"]})
        else:
            rparam.grad = res["dW_r"].clone()
            ropt.step()
            rparam.grad = None
        rec = {"y": res["y"], "dX": res["dX"], "dW_r": res["dW_r"], "weights": res["weights"],
               "logits": res["logits"], "compact": {n: store.compact[n].clone() for n in shapes},
               "master_after": {n: masters[n].clone() for n in shapes},
               "w_r_after": w_r.clone()}
        if router == "sgd":
            rec["momentum"] = ropt.state[rparam]["momentum_buffer"].clone()
        out.append(rec)
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
