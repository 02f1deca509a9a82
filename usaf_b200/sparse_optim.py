"""SparseAdam with device-resident state (usaf/sparse_optim.py:4-188).

Same constructor, methods and properties as the reference.  ``m``/``v`` live
on the parameter's CUDA device; ``step`` is one fused kernel per tensor
(``usaf_sparse_adam`` in compact mode, ``usaf_sparse_adam_gather`` otherwise).
When a compact master is registered with a :class:`Projection` via
``bind_projection``, the same kernel writes the new fp16-rounded values into
the GEMM overlay (``sync_resident`` fused in).  ``state_dict`` returns CPU
tensors so checkpoints keep the reference's format.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch

from . import engine


class SparseAdam:
    def __init__(self, named_params: Dict[str, torch.nn.Parameter],
                 active_mask: Optional[Dict[str, torch.Tensor]] = None,
                 active_idx: Optional[Dict[str, torch.Tensor]] = None, lr: float = 1e-4,
                 betas: tuple = (0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.01,
                 compact_params: bool = False):
        self.compact_params = compact_params
        self.lr = lr
        self.betas = betas
        self.eps = eps
        self.weight_decay = weight_decay
        self._named = dict(named_params)
        self._step = 0
        self._proj: Dict[str, engine.Projection] = {}
        if active_idx is not None:
            self._build_state_from_idx(active_idx)
        else:
            self._build_state(active_mask or {})

    def _dev(self, name):
        p = self._named[name]
        if not p.is_cuda:
            raise TypeError("usaf_b200 SparseAdam keeps its state on the parameter's CUDA device")
        return p.device

    def _check_idx(self, name, idx):
        """The kernels index the parameter (gather/scatter mode) or its gradient
        with ``idx``; an entry outside them is refused here, where the
        reference's own torch indexing would raise IndexError in ``step``."""
        lo, hi = int(idx.min()), int(idx.max())
        if lo < 0 or (not self.compact_params and hi >= self._named[name].numel()):
            raise IndexError(f"{name}: active index out of range")
        self._idx_max[name] = hi

    def _build_state_from_idx(self, active_idx):
        self._active_ids, self._idx, self._m, self._v = [], {}, {}, {}
        self._idx_max: Dict[str, int] = {}
        for name, idx in active_idx.items():
            if name not in self._named or idx is None or idx.numel() == 0:
                continue
            dev = self._dev(name)
            idx = idx.reshape(-1).to(device=dev, dtype=torch.long)
            self._check_idx(name, idx)
            self._active_ids.append(name)
            self._idx[name] = idx
            self._m[name] = torch.zeros(idx.numel(), device=dev, dtype=torch.float32)
            self._v[name] = torch.zeros(idx.numel(), device=dev, dtype=torch.float32)

    def _build_state(self, active_mask):
        self._active_ids, self._idx, self._m, self._v = [], {}, {}, {}
        self._idx_max: Dict[str, int] = {}
        for name in self._named:
            mask = active_mask.get(name)
            if mask is None:
                continue
            dev = self._dev(name)
            idx = mask.reshape(-1).to(device=dev, dtype=torch.bool).nonzero().reshape(-1)
            if idx.numel() == 0:
                continue
            self._check_idx(name, idx)
            self._active_ids.append(name)
            self._idx[name] = idx
            self._m[name] = torch.zeros(idx.numel(), device=dev, dtype=torch.float32)
            self._v[name] = torch.zeros(idx.numel(), device=dev, dtype=torch.float32)

    def bind_projection(self, name: str, proj: engine.Projection) -> None:
        """Let ``step`` write ``name``'s new values into ``proj``'s overlay."""
        self._proj[name] = proj

    def zero_grad(self, set_to_none: bool = False):
        for name in self._active_ids:
            p = self._named[name]
            if p.grad is not None:
                if set_to_none:
                    p.grad = None
                else:
                    p.grad.zero_()

    def step(self, compact_grads: Optional[Dict[str, torch.Tensor]] = None, grad_div: float = 1.0):
        """One Adam step over the active elements (usaf/sparse_optim.py:86-134).

        ``grad_div`` divides the gradients first (train.py:661-662 passes
        ``compact / (loss_scale*ACCUM)``; here the division is fused)."""
        self._step += 1
        for name in self._active_ids:
            p = self._named[name]
            if compact_grads is None and p.grad is None:
                continue
            if compact_grads is not None:
                g = compact_grads.get(name)
                if g is None:
                    continue
                g = g.detach().to(device=p.device, dtype=torch.float32).contiguous()
                if self.compact_params:
                    engine.sparse_adam_compact(p.data, self._m[name], self._v[name], g,
                                               self._step, self.lr, self.betas, self.eps,
                                               self.weight_decay, proj=self._proj.get(name),
                                               grad_div=grad_div,
                                               dtype=self._proj[name].dtype if name in self._proj else torch.float32)
                    continue
                dense = torch.zeros(p.numel(), device=p.device, dtype=p.dtype)
                dense[self._idx[name]] = g.to(p.dtype)
                grad = dense
            else:
                grad = p.grad.detach().reshape(-1).contiguous()
                if self._idx_max[name] >= grad.numel():
                    raise IndexError(f"{name}: active index out of range of its gradient")
            if self.compact_params:
                engine.sparse_adam_compact(p.data, self._m[name], self._v[name],
                                           grad.float().index_select(0, self._idx[name]),
                                           self._step, self.lr, self.betas, self.eps,
                                           self.weight_decay, grad_div=grad_div)
            else:
                engine.sparse_adam_gather(p.data, grad, self._idx[name], self._m[name],
                                          self._v[name], self._step, self.lr, self.betas,
                                          self.eps, self.weight_decay, grad_div=grad_div)

    def refresh(self, model):
        current = dict(model.named_parameters())
        for name in self._active_ids:
            if name in current and current[name].numel() == self._named[name].numel():
                self._named[name] = current[name]

    def reselect(self, named_params, new_active_mask):
        self._named = dict(named_params)
        self._build_state(new_active_mask)

    def state_dict(self) -> dict:
        return {"step": self._step,
                "m": {n: t.detach().cpu().clone() for n, t in self._m.items()},
                "v": {n: t.detach().cpu().clone() for n, t in self._v.items()}}

    def load_state_dict(self, sd: dict) -> None:
        self._step = int(sd["step"])
        for n, t in sd["m"].items():
            if n in self._m and t.numel() == self._m[n].numel():
                self._m[n] = t.detach().reshape(-1).to(self._m[n].device).float().clone()
        for n, t in sd["v"].items():
            if n in self._v and t.numel() == self._v[n].numel():
                self._v[n] = t.detach().reshape(-1).to(self._v[n].device).float().clone()

    @property
    def num_active_params(self) -> int:
        return sum(idx.numel() for idx in self._idx.values())

    @property
    def optimizer_memory_mb(self) -> float:
        return sum(self._m[n].numel() * 8 for n in self._active_ids) / (1024 * 1024)
