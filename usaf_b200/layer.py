"""One MoE layer's sparse training step on the device, in train.py's order.

importance pass -> ``TopKImportanceStore.select(frac)`` (train.py:397-402) ->
fp32 masters from the original int4 dequant (train.py:451-467) -> training
passes with ``SparseGradStore`` capture (train.py:631-641) -> SparseAdam over
the masters (compact) and the router (train.py:490, 665) -> RigL merge every
``reselect_every`` steps (train.py:536-613).
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

from . import engine
from .engine import BlockDims, MoEBlock, Projection
from .moe_loader import SparseGradStore, TopKImportanceStore
from .sparse_optim import SparseAdam
from . import rigl


class SparseMoELayer:
    def __init__(self, w_r: torch.Tensor, gate_up: Projection, down: Projection, top_k: int,
                 T: int, norm_topk_prob: bool = True, prefix: str = "layer.mlp.experts",
                 pair_factor: int = 2):
        E, H = w_r.shape
        I = down.C
        self.dtype = w_r.dtype
        self.w_r = w_r
        self.gu, self.dn = gate_up, down
        self.prefix = prefix
        self.names = {f"{prefix}.gate_up_proj": gate_up, f"{prefix}.down_proj": down}
        self.shapes = {n: p.shape for n, p in self.names.items()}
        self.block = MoEBlock(BlockDims(T, H, E, I, top_k, norm_topk_prob, w_r.dtype),
                              w_r.device, pair_factor)
        self.active: Dict[str, torch.Tensor] = {}
        self.masters: Dict[str, torch.Tensor] = {}
        self.store: Optional[SparseGradStore] = None
        self.opt: Optional[SparseAdam] = None
        self.router_opt: Optional[SparseAdam] = None

    # -------------------------------------------------------------------
    def forward_backward(self, x, dy):
        y = self.block.forward(x, self.w_r, self.gu, self.dn)
        dx, dw_r = self.block.backward(dy, x, self.w_r, self.gu, self.dn)
        return y, dx, dw_r

    def importance(self, x, dy, frac: float, cand_mult: float = 2.0) -> TopKImportanceStore:
        store = TopKImportanceStore(self.shapes, frac, cand_mult)
        self.forward_backward(x, dy)
        for name, p in self.names.items():
            store.add_from(name, self.block, name.rsplit(".", 1)[1])
        return store

    def init_selection(self, active: Dict[str, torch.Tensor], lr=1e-4, weight_decay=0.01,
                       router_lr=None, router_optimizer: str = "adam"):
        """Masters from the original int4 dequant at ``active``, overlays,
        capture store and the optimizers.  ``router_optimizer``: ``"adam"``
        steps the router with SparseAdam over all of W_r (the C2
        configuration); ``"sgd"`` with train.py's SGD, momentum 0.9 and the
        same weight decay (train.py:494-498, 667-672)."""
        # compact vectors (masters, moments, gradients) in CSR order: the kernels'
        # compact <-> overlay maps become the identity (streaming accesses)
        self.active = {n: a.reshape(-1).long() for n, a in active.items()}
        for name, p in self.names.items():
            if name in self.active:
                self.active[name] = self.active[name][p.csr_order(self.active[name])]
        self.masters = {}
        for name, p in self.names.items():
            deq = p.dequant(torch.float16).reshape(-1)
            self.masters[name] = deq.index_select(0, self.active[name]).float()
            p.set_overlay(self.active[name], self.masters[name])
        self.store = SparseGradStore(self.active, self.shapes)
        params = {n: torch.nn.Parameter(m, requires_grad=False) for n, m in self.masters.items()}
        self.opt = SparseAdam(params, active_idx=self.active, lr=lr,
                              weight_decay=weight_decay, compact_params=True)
        for name, p in self.names.items():
            self.opt.bind_projection(name, p)
        self.params = params
        E, H = self.w_r.shape
        rname = self.prefix.replace(".experts", ".gate.weight")
        self.router_name = rname
        self.router_param = torch.nn.Parameter(self.w_r, requires_grad=False)
        self.use_router_optimizer(router_optimizer, router_lr if router_lr is not None else lr,
                                  weight_decay)

    def use_router_optimizer(self, kind: str, lr: float, weight_decay: float = 0.01):
        """A fresh router optimizer: ``"adam"`` (SparseAdam over all of W_r) or
        ``"sgd"`` (train.py's SGD, momentum 0.9, train.py:494-498)."""
        if kind not in ("adam", "sgd"):
            raise ValueError(f"router optimizer must be 'adam' or 'sgd', got {kind!r}")
        E, H = self.w_r.shape
        self.router_sgd = self.router_opt = None
        if kind == "sgd":
            self.router_sgd = torch.optim.SGD([self.router_param], lr=lr, momentum=0.9,
                                              weight_decay=weight_decay)
        else:
            self.router_opt = SparseAdam({self.router_name: self.router_param},
                                         active_idx={self.router_name: torch.arange(E * H, device=self.w_r.device)},
                                         lr=lr, weight_decay=weight_decay)

    def train_step(self, x, dy, loss_scale: float = 1.0, accum: int = 1, micro=None):
        """One optimizer step over ``accum`` micro-batches (x, dy pairs)."""
        self.store.zero_()
        dw_r_acc = None
        pairs = micro if micro is not None else [(x, dy)]
        out = None
        for xm, dym in pairs:
            y, dx, dw_r = self.forward_backward(xm, dym)
            self.block.sparse_grads(self.gu, self.dn, self.store.compact[self._gu_name()],
                                    self.store.compact[self._dn_name()])
            dw_r_acc = dw_r.clone() if dw_r_acc is None else dw_r_acc.add_(dw_r)
            out = (y, dx, dw_r)
        denom = float(loss_scale * accum)
        self.opt.step(compact_grads=self.store.compact, grad_div=denom)
        self.router_param.grad = dw_r_acc
        if self.router_sgd is not None:
            # train.py:667-671: the gradient is divided in place, then SGD steps
            dw_r_acc.div_(denom)
            self.router_sgd.step()
        else:
            self.router_opt.step(grad_div=denom)
        self.router_param.grad = None
        return out

    def reselect(self, x, dy, frac: float, lr=None):
        """RigL merge (train.py:536-613) with a fresh optimizer."""
        store = self.importance(x, dy, frac)
        new_idx = store.select(frac)
        new_active, new_masters = {}, {}
        for name, p in self.names.items():
            orig = p.dequant(torch.float16).reshape(-1)
            fin, vals = rigl.merge(self.active[name], new_idx.get(name), self.masters[name], orig)
            new_active[name], new_masters[name] = fin, vals
        lr = self.opt.lr if lr is None else lr
        self.init_selection_from(new_active, new_masters, lr)
        return new_active

    def init_selection_from(self, active, masters, lr, weight_decay=0.01):
        self.active, self.masters = {}, {}
        for name, a in active.items():
            perm = self.names[name].csr_order(a) if name in self.names else None
            self.active[name] = a.long() if perm is None else a.long()[perm]
            self.masters[name] = masters[name] if perm is None else masters[name][perm]
        for name, p in self.names.items():
            p.set_overlay(self.active[name], self.masters[name])
        self.store = SparseGradStore(self.active, self.shapes)
        params = {n: torch.nn.Parameter(m, requires_grad=False) for n, m in self.masters.items()}
        self.opt = SparseAdam(params, active_idx=self.active, lr=lr, weight_decay=weight_decay,
                              compact_params=True)
        for name, p in self.names.items():
            self.opt.bind_projection(name, p)
        self.params = params

    def reorder_to(self, name: str, vec: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
        """A compact vector of ``name`` (aligned with ``self.active[name]``, kept in
        CSR order) re-aligned with the caller's index list ``idx`` (same set)."""
        a = self.active[name]
        o_a = torch.argsort(a)
        o_i = torch.argsort(idx.reshape(-1).to(device=a.device, dtype=torch.long))
        out = torch.empty_like(vec)
        out[o_i] = vec[o_a]
        return out

    def _gu_name(self):
        return f"{self.prefix}.gate_up_proj"

    def _dn_name(self):
        return f"{self.prefix}.down_proj"
