"""Step driver of sparse expert training over the patched Qwen3-MoE path.

The loop semantics are train.py's (the reference trains through its own
script body; this is the same loop as a class over a model patched with
:func:`usaf_b200.qwen3moe.patch_qwen3moe_for_b200` whose experts carry int4
weights from :func:`usaf_b200.qwen3moe.attach_int4_experts`):

* learning rate (train.py:500, 617-624): linear warm-up to ``lr_peak`` over
  ``max(1, int(steps * 0.05))`` steps, then cosine decay to
  ``lr_min = lr_peak / 10``; applied to the expert SparseAdam and the router
  optimizer;
* dynamic loss scale (train.py:31, 234, 351-353, 661-677): every micro-batch
  backpropagates ``loss * loss_scale``; the expert gradients (and the router
  gradients) are divided by ``loss_scale * accum`` before the step; a step
  whose expert gradients hold inf/nan is skipped (no optimizer update) and
  halves the scale (floor 64); every ``scale_up_every`` consecutive good steps
  double it (cap 65536);
* accumulation (train.py:634-641): ``accum`` micro-batches per step, the
  gradient store zeroed once per step, the logged loss the micro-batch mean;
* RigL reselection (train.py:625-629, 536-613): at every step > 1 that is a
  multiple of ``reselect_every``, before its micro-batches: one dense
  importance pass on the step's first micro-batch, the kept/grown merge of
  :func:`usaf_b200.rigl.merge`, fresh SparseAdam state;
* router optimizer (train.py:494-498, 667-672): SGD with momentum 0.9 and the
  same weight decay over the gate weights of the blocks whose experts train;
* experts sharded over ranks (``attach_int4_experts(..., expert_parallel=True)``):
  every rank trains its shard's coordinates, the importance selection is the
  per-tensor top-k over all ranks' candidates (the single-process selection
  over the union of the ranks' batches), the router gradient is summed over
  the ranks, and every rank takes the same skip / raise decision; each rank
  saves its own checkpoint file.  A step over W ranks with ``accum``
  micro-batches each is one process accumulating ``accum * W`` micro-batches:
  the summed gradients are divided by ``loss_scale * accum * W``.

Everything stays on the device; one host read per step carries the
finiteness flag, the loss and the error words of the block workspaces (a
batch whose routed pairs exceed a workspace raises ``UsafError`` there,
before any update).
"""
from __future__ import annotations

import math
from typing import Any, Callable, Dict, Iterable, List, Optional

import torch
import torch.distributed as dist

from . import checkpoint as ckpt
from . import qwen3moe, rigl
from ._lib import UsafError
from .engine import Projection
from .expert_parallel import global_select
from .moe_loader import SparseGradStore, TopKImportanceStore
from .sparse_optim import SparseAdam

LOSS_SCALE_INIT = 4096.0      # train.py:31
SCALE_UP_EVERY = 200          # train.py:31
LOSS_SCALE_MAX = 65536.0      # train.py:674
LOSS_SCALE_MIN = 64.0         # train.py:676


def lr_at(step: int, steps: int, lr_peak: float, lr_min: Optional[float] = None) -> float:
    """train.py:617-624 (warm-up = max(1, int(steps * 0.05)), lr_min = lr_peak / 10)."""
    warmup = max(1, int(steps * 0.05))
    lr_min = lr_peak / 10 if lr_min is None else lr_min
    if step <= warmup:
        return lr_peak * step / warmup
    cos_lr = 0.5 * (1 + math.cos(math.pi * (step - warmup) / (steps - warmup)))
    return lr_min + (lr_peak - lr_min) * cos_lr


class LossScaler:
    """The loss-scale state machine of train.py:661-677."""

    def __init__(self, init: float = LOSS_SCALE_INIT, scale_up_every: int = SCALE_UP_EVERY):
        self.scale = float(init)
        self.scale_up_every = int(scale_up_every)
        self.good_streak = 0
        self.n_skipped = 0

    def update(self, finite: bool) -> None:
        if finite:
            self.good_streak += 1
            if self.good_streak % self.scale_up_every == 0:
                self.scale = min(self.scale * 2, LOSS_SCALE_MAX)
        else:
            self.n_skipped += 1
            self.scale = max(self.scale / 2, LOSS_SCALE_MIN)

    def state_dict(self) -> Dict[str, Any]:
        return {"loss_scale": self.scale, "good_streak": self.good_streak, "n_skipped": self.n_skipped}

    def load_state_dict(self, sd: Dict[str, Any]) -> None:
        self.scale = float(sd["loss_scale"])
        self.good_streak = int(sd.get("good_streak", 0))
        self.n_skipped = int(sd.get("n_skipped", 0))


LossFn = Callable[[torch.nn.Module, Any], torch.Tensor]


class SparseTrainer:
    """train.py's step loop over the int4 experts of ``model``.

    ``loss_fn(model, micro_batch)`` runs the forward and returns the scalar
    loss; the trainer runs the backward of ``loss * loss_scale``."""

    def __init__(self, model: torch.nn.Module, steps: int, lr_peak: float = 2e-4,
                 weight_decay: float = 0.005, accum: int = 1, frac: float = 0.005,
                 reselect_every: int = 50, loss_scale_init: float = LOSS_SCALE_INIT,
                 scale_up_every: int = SCALE_UP_EVERY, train_router: bool = True,
                 expert_names: Optional[Iterable[str]] = None):
        """``expert_names``: the ``*.mlp.experts`` modules to train (default:
        every one with int4 weights attached); the others run frozen."""
        self.model = model
        self.steps, self.lr_peak, self.weight_decay = int(steps), float(lr_peak), float(weight_decay)
        self.accum, self.frac, self.reselect_every = int(accum), float(frac), int(reselect_every)
        wanted = set(expert_names) if expert_names is not None else None
        self.experts: Dict[str, torch.nn.Module] = {
            n: m for n, m in model.named_modules()
            if n.endswith(".mlp.experts") and getattr(m, "_usaf_int4", None) is not None
            and (wanted is None or n in wanted)}
        if not self.experts:
            raise ValueError("no experts with int4 weights attached (attach_int4_experts)")
        self.projections: Dict[str, Projection] = {}
        for n, m in self.experts.items():
            gu, dn = m._usaf_int4
            self.projections[f"{n}.gate_up_proj"] = gu
            self.projections[f"{n}.down_proj"] = dn
        self.shapes = {n: p.shape for n, p in self.projections.items()}
        # experts sharded over ranks (attach_int4_experts(..., expert_parallel=True)):
        # the projections are this rank's shards; selection runs over the full tensors
        ep = {bool(getattr(m, "_usaf_ep", False)) for m in self.experts.values()}
        if len(ep) > 1:
            raise ValueError("either every expert module is sharded over ranks or none is")
        self.expert_parallel = ep == {True}
        self.ep_group = (next(iter(self.experts.values()))._usaf_ep_group
                         if self.expert_parallel else None)
        if self.expert_parallel:
            W = dist.get_world_size(self.ep_group)
            self.ep_rank = dist.get_rank(self.ep_group)
            self.full_shapes = {n: (sh[0] * W,) + tuple(sh[1:]) for n, sh in self.shapes.items()}
        self.router_params: Dict[str, torch.nn.Parameter] = {}
        if train_router:
            for n in self.experts:
                blk = model.get_submodule(n.rsplit(".", 1)[0])
                self.router_params[f"{n.rsplit('.', 1)[0]}.gate.weight"] = blk.gate.weight
        self.router_opt = (torch.optim.SGD(list(self.router_params.values()), lr=self.lr_peak,
                                           momentum=0.9, weight_decay=self.weight_decay)
                           if self.router_params else None)
        self.scaler = LossScaler(loss_scale_init, scale_up_every)
        self.step_num = 0
        self.losses: List[float] = []
        self.active: Dict[str, torch.Tensor] = {}
        self.masters: Dict[str, torch.nn.Parameter] = {}
        self.store: Optional[SparseGradStore] = None
        self.opt: Optional[SparseAdam] = None

    # ---------------------------------------------------------------- capture
    def _set_capture(self, store) -> None:
        for n, m in self.experts.items():
            m._grad_capture = (store, n)

    def _backward(self, loss_fn: LossFn, batch) -> torch.Tensor:
        loss = loss_fn(self.model, batch)
        (loss * self.scaler.scale).backward()
        return loss.detach().float()

    # -------------------------------------------------------------- selection
    def importance(self, batch, loss_fn: LossFn) -> Dict[str, torch.Tensor]:
        """Dense importance pass (train.py:386-402, 540-546): the top ``frac`` of
        |dW| per tensor on one micro-batch."""
        store = TopKImportanceStore(self.full_shapes if self.expert_parallel else self.shapes,
                                    frac=self.frac)
        self._set_capture(store)
        try:
            self._backward(loss_fn, batch)
        finally:
            self._set_capture(self.store) if self.store is not None else self._clear_capture()
        for p in self.router_params.values():
            p.grad = None
        if not self.expert_parallel:
            return store.select(self.frac)
        # per full tensor: top-k over every rank's candidates, then this rank's share
        # as flat indices of its shard
        dev = next(iter(self.projections.values())).device
        out: Dict[str, torch.Tensor] = {}
        for name, shape in self.full_shapes.items():
            vals, idxs = store.candidate_list(name, device=dev)
            k = max(1, int(math.prod(shape) * self.frac))
            g = global_select(vals, idxs, k, self.ep_group)
            out[name] = shard_share(g, self.ep_rank, math.prod(self.shapes[name]))
        return out

    def _clear_capture(self) -> None:
        for m in self.experts.values():
            if hasattr(m, "_grad_capture"):
                del m._grad_capture

    def init_selection(self, active_idx: Dict[str, torch.Tensor],
                       masters: Optional[Dict[str, torch.Tensor]] = None, lr: Optional[float] = None,
                       optimizer_state: Optional[dict] = None) -> None:
        """Masters from the original int4 dequant (fp16 -> fp32) unless given
        (train.py:451-467), overlays installed, capture store and a fresh
        SparseAdam (train.py:490, 600-610)."""
        self.active, self.masters = {}, {}
        for name, p in self.projections.items():
            if name not in active_idx:
                continue
            a = active_idx[name].reshape(-1).to(device=p.device, dtype=torch.long)
            perm = p.csr_order(a)     # compact vectors in CSR order (streaming overlay maps)
            a = a[perm]
            if masters is not None and name in masters:
                m = masters[name].reshape(-1).to(device=p.device, dtype=torch.float32)[perm]
            else:
                m = p.dequant(torch.float16).reshape(-1).index_select(0, a).float()
            self.active[name] = a
            self.masters[name] = torch.nn.Parameter(m, requires_grad=False)
            p.set_overlay(a, m)
            if optimizer_state is not None:
                optimizer_state = _permute_state(optimizer_state, name, perm)
        self.store = SparseGradStore(self.active, self.shapes)
        self._set_capture(self.store)
        self.opt = SparseAdam(self.masters, active_idx=self.active,
                              lr=self.lr_peak if lr is None else lr,
                              weight_decay=self.weight_decay, compact_params=True)
        for name in self.active:
            self.opt.bind_projection(name, self.projections[name])
        if optimizer_state is not None:
            self.opt.load_state_dict(optimizer_state)

    def reselect(self, batch, loss_fn: LossFn, lr: float) -> None:
        """RigL merge (train.py:536-613)."""
        new_idx = self.importance(batch, loss_fn)
        fin_a, fin_m = {}, {}
        for name, p in self.projections.items():
            if name not in self.active:
                continue
            orig = p.dequant(torch.float16).reshape(-1)
            fin_a[name], fin_m[name] = rigl.merge(self.active[name], new_idx.get(name),
                                                  self.masters[name].data, orig)
        self.init_selection(fin_a, fin_m, lr=lr)

    # ------------------------------------------------------------------- step
    def train_step(self, micro_batches: Iterable, loss_fn: LossFn) -> Dict[str, Any]:
        if self.opt is None:
            raise RuntimeError("init_selection() first")
        micro_batches = list(micro_batches)
        if len(micro_batches) != self.accum:
            raise ValueError(f"expected {self.accum} micro-batches, got {len(micro_batches)}")
        self.step_num += 1
        step = self.step_num
        lr = lr_at(step, self.steps, self.lr_peak)
        self.opt.lr = lr
        if step > 1 and step % self.reselect_every == 0:
            self.reselect(micro_batches[0], loss_fn, lr)
        if self.router_opt is not None:
            for pg in self.router_opt.param_groups:
                pg["lr"] = lr
            self.router_opt.zero_grad()
        self.store.zero_()
        loss_sum = torch.zeros((), dtype=torch.float32, device=next(iter(self.masters.values())).device)
        for mb in micro_batches:
            loss_sum += self._backward(loss_fn, mb)
        scale = self.scaler.scale
        # train.py:661-662 divides the summed gradients by loss_scale * ACCUM.  Under
        # expert parallelism every shard's gradient (and the all-reduced router
        # gradient) sums W ranks' micro-batches, each with a loss averaged over its
        # own tokens: one step is one process accumulating accum * W micro-batches
        denom = scale * self.accum * (dist.get_world_size(self.ep_group) if self.expert_parallel else 1)
        # train.py:662-663: the step runs only if every expert gradient is finite
        flags = torch.stack([torch.isfinite(g).all() for g in self.store.compact.values()])
        blocks = qwen3moe.workspaces(self.model)
        nf = flags.numel()
        dev_vals = torch.cat([flags.float(), loss_sum.reshape(1)] + [b.err.float() for b in blocks])
        if self.expert_parallel:
            dev_vals = ranks_agree(dev_vals, nf, self.ep_group)
        host = dev_vals.cpu()
        if bool(host[nf + 1:].any()):
            for b in blocks:
                b.err.zero_()
            self.step_num -= 1
            raise UsafError("a block workspace reported a device error in this step (routed "
                            "pairs beyond its buffer, or a timed-out wait); no update applied")
        finite = bool(host[:nf].all())
        if finite:
            self.opt.step(compact_grads=self.store.compact, grad_div=denom)
            if self.router_opt is not None:
                for p in self.router_params.values():
                    if p.grad is not None:
                        p.grad.data.div_(denom)
                self.router_opt.step()
                self.router_opt.zero_grad()
        elif self.router_opt is not None:
            self.router_opt.zero_grad()
        self.scaler.update(finite)
        loss = float(host[nf]) / self.accum
        self.losses.append(loss)
        return {"step": step, "loss": loss, "lr": lr, "scale": self.scaler.scale,
                "finite": finite}

    # ------------------------------------------------------------- checkpoint
    def save_checkpoint(self, path: str, metric: Optional[float] = None) -> str:
        """usaf-sparse-v1 file (usaf/checkpoint.py:20-47); the loss-scale state
        goes into ``config``."""
        train_layers = sorted({int(n.split(".layers.")[1].split(".")[0])
                               for n in self.experts if ".layers." in n})
        config = {"lr_peak": self.lr_peak, "wd": self.weight_decay, "frac": self.frac,
                  "accum": self.accum, "steps": self.steps, **self.scaler.state_dict()}
        return ckpt.save_sparse_checkpoint(path, {n: m.data for n, m in self.masters.items()},
                                           self.active, self.opt.state_dict(), config,
                                           self.step_num, self.losses, train_layers, metric)

    def load_checkpoint(self, path: str) -> None:
        st = ckpt.load_sparse_checkpoint(path)
        self.step_num = int(st["step"])
        self.losses = list(st.get("losses", []))
        cfg = st.get("config") or {}
        if "loss_scale" in cfg:
            self.scaler.load_state_dict(cfg)
        lr = lr_at(max(self.step_num, 1), self.steps, self.lr_peak)
        self.init_selection(st["active_idx"], st["masters"], lr=lr, optimizer_state=st["optimizer"])


def shard_share(g: torch.Tensor, rank: int, span: int) -> torch.Tensor:
    """This rank's part of a global selection ``g`` (flat indices of the full
    [E, R, C] tensor) as flat indices of its shard: rank r owns the flat
    range [r * span, (r + 1) * span), span = (E / W) * R * C."""
    lo = rank * span
    return g[(g >= lo) & (g < lo + span)] - lo


def ranks_agree(dev_vals: torch.Tensor, nf: int, group=None) -> torch.Tensor:
    """One decision for all ranks of an expert-parallel step.

    ``dev_vals`` = ``nf`` finiteness flags (1 = finite) of this rank's expert
    gradients, the rank's summed loss, then the error words of its block
    workspaces.  Returns the same layout: a flag is 1 only if it is 1 on
    every rank (a non-finite shard skips the step everywhere), the loss is
    the ranks' mean, and the last entry counts the nonzero error words over
    all ranks (any of them makes every rank raise)."""
    agg = torch.cat([(1.0 - dev_vals[:nf]), dev_vals[nf:nf + 1],
                     (dev_vals[nf + 1:] != 0).float().sum().reshape(1)])
    dist.all_reduce(agg, group=group)
    W = dist.get_world_size(group)
    return torch.cat([(agg[:nf] == 0).float(), agg[nf:nf + 1] / W, agg[nf + 1:]])


def _permute_state(sd: dict, name: str, perm: torch.Tensor) -> dict:
    """Optimizer state of ``name`` re-ordered like its active list."""
    out = dict(sd)
    for key in ("m", "v"):
        if key in sd and name in sd[key]:
            out[key] = dict(sd[key])
            out[key][name] = sd[key][name].reshape(-1)[perm.cpu()]
    return out
