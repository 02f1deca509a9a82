"""train.py's sparse training loop restated on the CPU (test oracle only).

One optimizer step (train.py:616-677) over a Qwen3-MoE causal LM whose MoE
blocks compute the reference's block (usaf/qwen3moe_dml.py:67-86, experts
dense-masked, :24-64) with expert weights = fp16 int4 dequant with the
trained coordinates overlaid (``_get_resident`` after ``sync_resident``,
usaf/moe_loader.py:226-247, 425-443), rebuilt from the masters before every
forward:

* lr = warm-up + cosine (train.py:616-624) for the expert SparseAdam and the
  router SGD (train.py:494-498, 626-629);
* every micro-batch backpropagates ``loss * loss_scale`` (train.py:351);
  expert gradients go to a ``SparseGradStore`` through the capture hooks
  (train.py:408-412, 631-641), the router weights get their autograd
  gradients;
* the step divides by ``loss_scale * ACCUM``, runs only if every compact
  gradient is finite, then SparseAdam over the masters and SGD over the
  routers (train.py:661-672); the loss scale doubles every
  ``scale_up_every`` good steps and halves (floor 64) on a skipped one
  (train.py:673-677).

Helpers here only sequence the oracle's own restated pieces (oracle/moe.py).
"""
from __future__ import annotations

import math
import types
from typing import Dict, List

import numpy as np
import torch

from . import moe


def lr_at(step: int, steps: int, lr_peak: float) -> float:
    """train.py:616-624 (warm-up = max(1, int(steps * 0.05)), lr_min = lr_peak / 10)."""
    warm = max(1, int(steps * 0.05))
    if step <= warm:
        return lr_peak * step / warm
    cos_lr = 0.5 * (1 + math.cos(math.pi * (step - warm) / (steps - warm)))
    return lr_peak / 10 + (lr_peak - lr_peak / 10) * cos_lr


def _block_forward(self, hidden_states):
    """The reference's MoE block forward (usaf/qwen3moe_dml.py:67-86) on the
    block's current effective expert weights, with the capture hooks of the
    store set on the experts module."""
    b, s, h = hidden_states.shape
    hs = hidden_states.reshape(-1, h)
    _, _, _, weights = moe.router_forward(hs, self.gate.weight, self.gate.top_k,
                                          bool(self.gate.norm_topk_prob))
    cap = getattr(self.experts, "_oracle_capture", None)
    y = moe.experts_dense_masked(hs, weights, self.experts._oracle_w[0], self.experts._oracle_w[1],
                                 capture=cap[0].add if cap else None, prefix=cap[1] if cap else "")
    return y.reshape(b, s, h)


class OracleTrainer:
    """train.py's loop over ``model`` (a CPU Qwen3MoeForCausalLM).

    ``int4[name]`` is the fp16 dequant (numpy) of each expert tensor
    ``{layer}.mlp.experts.gate_up_proj`` / ``.down_proj``; ``active[name]``
    the trained flat indices."""

    def __init__(self, model, int4: Dict[str, np.ndarray], active: Dict[str, torch.Tensor],
                 steps: int, lr_peak: float, weight_decay: float, accum: int,
                 loss_scale: float = 4096.0, scale_up_every: int = 200):
        self.model, self.int4, self.steps, self.lr_peak = model, int4, steps, lr_peak
        self.wd, self.accum = weight_decay, accum
        self.scale, self.scale_up_every, self.good, self.step_num = loss_scale, scale_up_every, 0, 0
        self.active = {n: a.reshape(-1).long() for n, a in active.items()}
        self.masters = {n: torch.from_numpy(np.ascontiguousarray(int4[n])).reshape(-1)
                        .index_select(0, self.active[n]).float() for n in self.active}
        self.opt = moe.SparseAdam(self.masters, self.active, lr=lr_peak, weight_decay=weight_decay,
                                  compact_params=True)
        self.prefixes = sorted({n.rsplit(".", 1)[0] for n in self.active})
        self.gates = [model.get_submodule(p.rsplit(".", 1)[0]).gate.weight for p in self.prefixes]
        for g in self.gates:
            g.requires_grad_(True)
        self.router_opt = torch.optim.SGD(self.gates, lr=lr_peak, momentum=0.9, weight_decay=weight_decay)
        for p in self.prefixes:
            blk = model.get_submodule(p.rsplit(".", 1)[0])
            blk.forward = types.MethodType(_block_forward, blk)
        self.losses: List[float] = []

    def _sync_resident(self):
        """Effective expert weights from the current masters."""
        for p in self.prefixes:
            ex = self.model.get_submodule(p)
            ws = []
            for which in ("gate_up_proj", "down_proj"):
                n = f"{p}.{which}"
                w = moe.effective_weight(self.int4[n], self.active[n], self.masters[n])
                ws.append(w.float())
            ex._oracle_w = ws

    def train_step(self, micro_batches) -> Dict[str, float]:
        self.step_num += 1
        lr = lr_at(self.step_num, self.steps, self.lr_peak)
        self.opt.lr = lr
        for pg in self.router_opt.param_groups:
            pg["lr"] = lr
        store = moe.SparseGradStore(self.active, {n: tuple(self.int4[n].shape) for n in self.active})
        for p in self.prefixes:
            self.model.get_submodule(p)._oracle_capture = (store, p)
        self.router_opt.zero_grad()
        loss_sum = 0.0
        for ids in micro_batches:
            self._sync_resident()
            loss = self.model(input_ids=ids, labels=ids).loss
            (loss * self.scale).backward()
            loss_sum += float(loss.detach())
        denom = self.scale * self.accum
        cg = {n: v / denom for n, v in store.compact.items()}
        finite = all(bool(torch.isfinite(v).all()) for v in cg.values())
        if finite:
            self.opt.step(cg)
            for g in self.gates:
                if g.grad is not None:
                    g.grad.data.div_(denom)
            self.router_opt.step()
            self.router_opt.zero_grad()
            self.good += 1
            if self.good % self.scale_up_every == 0:
                self.scale = min(self.scale * 2, 65536.0)
        else:
            self.scale = max(self.scale / 2, 64.0)
            self.router_opt.zero_grad()
        loss = loss_sum / self.accum
        self.losses.append(loss)
        return {"step": self.step_num, "loss": loss, "lr": lr, "scale": self.scale, "finite": finite}
