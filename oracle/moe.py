"""MoE expert hot path restated on the CPU with torch (test oracle only).

Every function cites the reference lines it restates.  The float math uses
the same torch CPU operators the reference calls (``F.linear``, ``softmax``,
``topk``, ``index_add_`` ...), so the oracle reproduces the reference's
numerics, including its rounding points (bf16 logits, bf16 expert outputs,
fp32 combine, fp32 optimizer state).
"""
from __future__ import annotations

import math
from typing import Callable, Dict, Optional

import numpy as np
import torch
import torch.nn.functional as F


# ---------------------------------------------------------------- router ---
def router_forward(hs: torch.Tensor, w_r: torch.Tensor, top_k: int, norm_topk_prob: bool):
    """Router of ``dml_qwen3_moe_block_forward`` (usaf/qwen3moe_dml.py:72-83).

    Returns ``(logits, probs, mask, weights)``: logits in the activation
    dtype, fp32 softmax, the threshold mask ``probs >= kth`` (ties admit
    more than ``top_k`` experts) and the renormalised dense weights cast back
    to the activation dtype.
    """
    logits = F.linear(hs, w_r)                                           # :73
    probs = F.softmax(logits, dtype=torch.float, dim=-1)                 # :74
    with torch.no_grad():
        top_val, _ = torch.topk(probs, top_k, dim=-1)                    # :77
        thresh = top_val[:, -1:].clone()                                 # :78
        mask = (probs >= thresh).to(probs.dtype)                         # :79
    weights = probs * mask                                               # :80
    if norm_topk_prob:
        weights = weights / weights.sum(dim=-1, keepdim=True).clamp_min(1e-9)  # :82
    return logits, probs, mask, weights.to(hs.dtype)                    # :83


# --------------------------------------------------------------- experts ---
CaptureFn = Callable[[str, int, torch.Tensor], None]


def experts_dense_masked(hs, weights, w_gu, w_dn, capture: Optional[CaptureFn] = None,
                         prefix: str = ""):
    """``dml_qwen3_experts_forward`` (usaf/qwen3moe_dml.py:24-64).

    Every expert runs on every token; the per-expert 2-D weight slices are
    detached leaves whose gradient hooks call ``capture(name, ei, grad)``
    (the ``store.add`` protocol, :43-47).  The combine is an fp32 sum in
    ascending expert order (:62).
    """
    final = torch.zeros(hs.shape, dtype=torch.float32)                   # :26
    weights_t = weights.t().contiguous()                                 # :27
    do_cap = capture is not None and torch.is_grad_enabled()
    for ei in range(w_gu.shape[0]):                                      # :49
        wg = w_gu[ei].detach()
        wd = w_dn[ei].detach()
        if do_cap:
            wg.requires_grad_(True)
            wd.requires_grad_(True)
            wg.register_hook(_hook(capture, prefix + ".gate_up_proj", ei))
            wd.register_hook(_hook(capture, prefix + ".down_proj", ei))
        gu = F.linear(hs, wg)                                            # :58
        gate, up = gu.chunk(2, dim=-1)                                   # :59
        cur = F.silu(gate) * up                                          # :60
        cur = F.linear(cur, wd)                                          # :61
        final = final + cur.float() * weights_t[ei].float().unsqueeze(-1)  # :62
    return final.to(hs.dtype)                                            # :64


def _hook(capture, name, ei):
    def h(g):
        capture(name, ei, g)
    return h


def dispatch_indices(weights: torch.Tensor) -> Dict[str, torch.Tensor]:
    """Dispatch metadata of ``batched_sparse_experts_forward``
    (benchmarks/kaggle_t4_bench.py:293-306).

    Pairs are the nonzero entries of the dense weights in row-major
    (token-major) order; a *stable* argsort by expert puts each expert's
    tokens in ascending token order; ``offs`` is the exclusive cumsum of the
    per-expert counts and ``pos`` the slot inside the expert's segment.
    """
    E = weights.shape[1]
    tok_idx, exp_idx = torch.nonzero(weights, as_tuple=True)            # :293
    counts = torch.bincount(exp_idx, minlength=E)                        # :296
    order = torch.argsort(exp_idx, stable=True)                          # :298
    exp_s = exp_idx[order]
    tok_s = tok_idx[order]                                               # :299
    offs = torch.zeros(E, dtype=torch.long)
    offs[1:] = torch.cumsum(counts, 0)[:-1]                              # :300-301
    pos = torch.arange(exp_s.numel()) - offs[exp_s]                      # :302
    slot_of_pair = torch.empty_like(order)
    slot_of_pair[order] = torch.arange(order.numel())
    return {"tok_idx": tok_idx, "exp_idx": exp_idx, "counts": counts, "offs": offs,
            "order": order, "tok_sorted": tok_s, "exp_sorted": exp_s, "pos": pos,
            "slot_of_pair": slot_of_pair}


def experts_sparse_loop(hs, weights, w_gu, w_dn, capture: Optional[CaptureFn] = None,
                        prefix: str = ""):
    """``sparse_qwen3_experts_forward`` (benchmarks/kaggle_t4_bench.py:253-282).

    Each expert runs only on its routed tokens (``nonzero`` of its weight
    column, ascending token order) and the weighted outputs are
    ``index_add``-ed in ascending expert order.  Numerically the same
    combine order as the dense-masked loop.
    """
    N, Hd = hs.shape
    final = torch.zeros(N, Hd, dtype=torch.float32)                      # :255
    do_cap = capture is not None and torch.is_grad_enabled()
    for ei in range(w_gu.shape[0]):                                      # :264
        w_col = weights[:, ei]
        idx = torch.nonzero(w_col, as_tuple=False).reshape(-1)           # :266
        if idx.numel() == 0:
            continue
        x_e = hs.index_select(0, idx)                                    # :269
        wg = w_gu[ei].detach()
        wd = w_dn[ei].detach()
        if do_cap:
            wg.requires_grad_(True)
            wd.requires_grad_(True)
            wg.register_hook(_hook(capture, prefix + ".gate_up_proj", ei))
            wd.register_hook(_hook(capture, prefix + ".down_proj", ei))
        gu = F.linear(x_e, wg)                                           # :276
        gate, up = gu.chunk(2, dim=-1)
        cur = F.silu(gate) * up
        cur = F.linear(cur, wd)
        cur = cur.float() * w_col.index_select(0, idx).float().unsqueeze(-1)  # :280
        final = final.index_add(0, idx, cur)                             # :281
    return final.to(hs.dtype)


def experts_batched(hs, weights, w_gu, w_dn, capture: Optional[CaptureFn] = None,
                    prefix: str = ""):
    """``batched_sparse_experts_forward`` (benchmarks/kaggle_t4_bench.py:284-328).

    The routed pairs are grouped by expert (the dispatch of
    :func:`dispatch_indices`) into a zero-padded ``[E, cap, H]`` batch, cap =
    the largest expert count; two ``bmm`` run every expert at once; the
    weighted rows are ``index_add``-ed into an fp32 output (padding rows carry
    weight 0).  Capture: one hook per stacked weight tensor hands each
    expert's slice of the ``[E, *, *]`` gradient to ``capture`` (:310-318).
    """
    N, Hd = hs.shape
    E = w_gu.shape[0]
    tok_idx, exp_idx = torch.nonzero(weights, as_tuple=True)             # :293
    if tok_idx.numel() == 0:
        return torch.zeros(N, Hd, dtype=hs.dtype)
    counts = torch.bincount(exp_idx, minlength=E)
    cap = int(counts.max().item())
    order = torch.argsort(exp_idx, stable=True)
    exp_s, tok_s = exp_idx[order], tok_idx[order]
    offs = torch.zeros(E, dtype=torch.long)
    offs[1:] = torch.cumsum(counts, 0)[:-1]
    pos = torch.arange(exp_s.numel()) - offs[exp_s]
    pad_tok = torch.zeros(E, cap, dtype=torch.long)
    pad_w = torch.zeros(E, cap, dtype=weights.dtype)
    pad_tok[exp_s, pos] = tok_s
    pad_w[exp_s, pos] = weights[tok_s, exp_s]                            # :306-307
    x_b = hs[pad_tok]                                                    # :309
    wg, wd = w_gu.detach(), w_dn.detach()
    if capture is not None and torch.is_grad_enabled():
        def _all(name):
            def h(g):
                for ei in range(E):
                    capture(name, ei, g[ei])
            return h
        wg.requires_grad_(True)
        wd.requires_grad_(True)
        wg.register_hook(_all(prefix + ".gate_up_proj"))
        wd.register_hook(_all(prefix + ".down_proj"))
    gu = torch.bmm(x_b, wg.transpose(1, 2))                              # :319
    gate, up = gu.chunk(2, dim=-1)
    cur = F.silu(gate) * up
    cur = torch.bmm(cur, wd.transpose(1, 2))                             # :322
    cur = cur.float() * pad_w.float().unsqueeze(-1)
    final = torch.zeros(N, Hd, dtype=torch.float32)
    final = final.index_add(0, pad_tok.reshape(-1), cur.reshape(-1, Hd))  # :325-326
    return final.to(hs.dtype)


def block_step(hs, w_r, w_gu, w_dn, dY, top_k: int, norm_topk_prob: bool = True,
               capture: Optional[CaptureFn] = None, prefix: str = "layer",
               experts: str = "sparse"):
    """One forward + backward of the MoE block with router co-training.

    Forward = ``dml_qwen3_moe_block_forward`` (usaf/qwen3moe_dml.py:67-86)
    with the experts computed dense-masked (:24-64, ``experts="dense"``), by
    the reference's per-expert sparse loop (benchmarks/kaggle_t4_bench.py:
    253-282, ``experts="sparse"``) or by its batched dispatch (:284-328,
    ``experts="batched"``); backward
    is ``y.backward(dY)`` through both, as the recompute-backward of
    train.py:356-364 does for one layer.  Expert gradients go to ``capture``;
    the router gradient and dX are returned.
    """
    hs = hs.detach().clone().requires_grad_(True)
    w_r = w_r.detach().clone().requires_grad_(True)
    logits, probs, mask, weights = router_forward(hs, w_r, top_k, norm_topk_prob)
    fn = {"dense": experts_dense_masked, "sparse": experts_sparse_loop,
          "batched": experts_batched}[experts]
    y = fn(hs, weights, w_gu, w_dn, capture=capture, prefix=prefix)
    y.backward(dY)
    return {"y": y.detach(), "dX": hs.grad.detach(), "dW_r": w_r.grad.detach(),
            "logits": logits.detach(), "probs": probs.detach(), "mask": mask,
            "weights": weights.detach()}


# ---------------------------------------------------------------- stores ---
class SparseGradStore:
    """Restates ``SparseGradStore`` (usaf/moe_loader.py:527-581): compact fp32
    gradients aligned with ``active_idx``; ``add`` gathers the dense
    per-expert gradient at the active local indices (:577) and index-adds it
    at the compact positions (:578)."""

    def __init__(self, active_idx, shapes):
        self.compact, self._maps = {}, {}
        for name, idx in active_idx.items():
            idx = idx.reshape(-1).to(dtype=torch.long)
            self.compact[name] = torch.zeros(idx.numel(), dtype=torch.float32)
            slice_size = int(np.prod([int(s) for s in shapes[name][1:]]))
            e_of = torch.div(idx, slice_size, rounding_mode="floor")
            per = {}
            for ei in torch.unique(e_of).tolist():
                pos = (e_of == ei).nonzero(as_tuple=False).reshape(-1)
                per[int(ei)] = (idx[pos] - ei * slice_size, pos)
            self._maps[name] = per

    def zero_(self):
        for v in self.compact.values():
            v.zero_()

    def add(self, full_name, ei, g):
        per = self._maps.get(full_name)
        if not per or int(ei) not in per:
            return
        local, pos = per[int(ei)]
        vals = g.detach().reshape(-1).gather(0, local).float()
        self.compact[full_name].index_add_(0, pos, vals)


class TopKImportanceStore:
    """Restates ``TopKImportanceStore`` (usaf/moe_loader.py:584-631).

    ``add`` keeps the top ``max(1, int(numel_e * frac * cand_mult))`` of
    ``|g|`` per expert slice (:604-611); ``select`` takes, per tensor, the top
    ``min(max(1, int(numel * frac)), n_candidates)`` of the union (:613-628),
    returned in descending-score order.
    """

    def __init__(self, shapes, frac, cand_mult=2.0):
        self._shapes, self._frac, self._cand = shapes, frac, cand_mult
        self._vals = {n: {} for n in shapes}
        self._idx = {n: {} for n in shapes}

    def zero_(self):
        for n in self._vals:
            self._vals[n].clear()
            self._idx[n].clear()

    def add(self, full_name, ei, g):
        if full_name not in self._vals:
            return
        flat = g.detach().float().reshape(-1).abs()
        k = max(1, int(flat.numel() * self._frac * self._cand))
        v, i = torch.topk(flat, min(k, flat.numel()))
        self._vals[full_name][int(ei)] = v
        self._idx[full_name][int(ei)] = i.to(torch.long) + int(ei) * flat.numel()

    def candidates(self, name):
        return dict(self._vals[name]), dict(self._idx[name])

    def select(self, frac=None):
        frac = self._frac if frac is None else frac
        out = {}
        for name, shape in self._shapes.items():
            if not self._vals[name]:
                continue
            vals = torch.cat(list(self._vals[name].values()))
            idxs = torch.cat(list(self._idx[name].values()))
            numel = int(np.prod([int(s) for s in shape]))
            k = min(max(1, int(numel * frac)), vals.numel())
            top = torch.topk(vals, k).indices
            out[name] = idxs[top]
        return out


# ------------------------------------------------------------- optimizer ---
def sparse_adam_update(p_active, m, v, grad, step, lr=1e-4, betas=(0.9, 0.999),
                       eps=1e-8, weight_decay=0.01):
    """One ``SparseAdam.step`` over a compact vector (usaf/sparse_optim.py:86-134).

    ``p_active`` is the fp32 view of the active values (the compact master,
    or the gathered parameter); ``m``/``v`` are updated in place.  Returns the
    fp32 ``delta`` (``-lr * update``, :127) that the caller adds to the
    parameter in its own dtype.  ``step`` is the post-increment step count.
    """
    beta1, beta2 = betas
    bias1 = 1 - beta1 ** step                                            # :96
    bias2 = 1 - beta2 ** step                                            # :97
    grad = grad.detach().to(torch.float32)
    if weight_decay > 0:
        grad = grad + weight_decay * p_active                            # :119
    m.mul_(beta1).add_(grad, alpha=1 - beta1)                            # :123
    v.mul_(beta2).addcmul_(grad, grad, value=1 - beta2)                  # :124
    update = (m / bias1) / ((v / bias2).sqrt() + eps)                    # :126
    return -lr * update                                                  # :127


class SparseAdam:
    """State-holding wrapper over :func:`sparse_adam_update` with the two
    parameter modes of usaf/sparse_optim.py: ``compact_params`` (the param is
    the 1-D master, :129-130) and gather/scatter (:131-134)."""

    def __init__(self, named_params, active_idx, lr=1e-4, betas=(0.9, 0.999), eps=1e-8,
                 weight_decay=0.01, compact_params=False):
        self.named, self.lr, self.betas, self.eps = dict(named_params), lr, betas, eps
        self.wd, self.compact, self._step = weight_decay, compact_params, 0
        self.idx = {n: i.reshape(-1).long() for n, i in active_idx.items()
                    if n in self.named and i.numel()}
        self.m = {n: torch.zeros(i.numel()) for n, i in self.idx.items()}
        self.v = {n: torch.zeros(i.numel()) for n, i in self.idx.items()}

    def step(self, grads):
        """``grads[name]``: compact fp32 grads (compact mode) or the dense
        parameter gradient (gather mode)."""
        self._step += 1
        for name, idx in self.idx.items():
            p = self.named[name]
            g = grads.get(name)
            if g is None:
                continue
            if self.compact:
                p_act = p.detach().float()
                grad = g.float()
            else:
                p_act = p.detach().reshape(-1).index_select(0, idx).float()
                grad = g.detach().reshape(-1).index_select(0, idx).float()
            delta = sparse_adam_update(p_act, self.m[name], self.v[name], grad, self._step,
                                       self.lr, self.betas, self.eps, self.wd)
            delta = delta.to(p.dtype)
            with torch.no_grad():
                if self.compact:
                    p.add_(delta)
                else:
                    flat = p.reshape(-1)
                    flat.scatter_(0, idx, flat.gather(0, idx) + delta)


# ------------------------------------------------------------- selectors ---
def kth_largest_threshold(scores: Dict[str, torch.Tensor], k: int) -> float:
    """``_kth_largest_threshold`` (usaf/selector.py:6-14)."""
    cat = torch.cat([s.reshape(-1) for s in scores.values()])
    n = cat.numel()
    k = max(1, min(k, n))
    arr = cat.numpy()
    kth = n - k
    return float(np.partition(arr, kth)[kth])


def topk_select(scores, k):
    """``TopKSelector.select`` (usaf/selector.py:21-25): ties are inclusive."""
    if not scores:
        return {}
    thr = kth_largest_threshold(scores, k)
    return {n: (s >= thr) for n, s in scores.items()}


def threshold_select(scores, percentile):
    """``ThresholdSelector.select`` (usaf/selector.py:32-39)."""
    cat = torch.cat([s.reshape(-1) for s in scores.values()])
    n = cat.numel()
    idx = min(max(int(n * percentile / 100.0), 0), n - 1)
    thr = float(np.partition(cat.numpy(), idx)[idx])
    return {name: (s >= thr) for name, s in scores.items()}


# ------------------------------------------------------------------ RigL ---
def rigl_merge(old: torch.Tensor, new: Optional[torch.Tensor], old_masters: torch.Tensor,
               original_flat: torch.Tensor):
    """Per-tensor RigL merge of ``do_reselect`` (train.py:552-596).

    ``kept = sorted(old & new)``, ``grown = sorted(new - old)[:len(old)-len(kept)]``,
    ``final = kept + grown`` (:560-565).  Kept coordinates keep their trained
    master (:575-583); grown ones restart from the ORIGINAL int4 dequant
    (``original_flat``, fp16, :585-593).  Returns ``(final_idx, new_masters)``.
    """
    if new is None or new.numel() == 0:
        return old.clone(), old_masters.clone()
    old_list = old.reshape(-1).tolist()
    old_set = set(old_list)
    nw_set = set(new.reshape(-1).tolist())
    kept = sorted(old_set & nw_set)
    candidates = sorted(nw_set - old_set)
    fill = max(0, len(old_set) - len(kept))
    grown = candidates[:fill]
    final = torch.tensor(kept + grown, dtype=torch.long)
    pos_of = {g: p for p, g in enumerate(old_list)}
    vals = torch.zeros(final.numel(), dtype=torch.float32)
    nk = len(kept)
    if nk:
        vals[:nk] = old_masters.float()[torch.tensor([pos_of[g] for g in kept])]
    if grown:
        vals[nk:] = original_flat.reshape(-1)[torch.tensor(grown)].float()
    return final, vals


# ----------------------------------------------------- effective weights ---
def effective_weight(dequant_fp16: np.ndarray, overlay_idx=None, overlay_vals=None):
    """Dequantized fp16 weight with overlays scattered in
    (usaf/moe_loader.py:241-247 ``_get_resident``; the master is rounded to
    fp16 exactly as ``sync_resident`` does, :442).  Returns a torch fp16 tensor."""
    t = torch.from_numpy(np.ascontiguousarray(dequant_fp16)).clone()
    if overlay_idx is not None:
        t.reshape(-1).scatter_(0, overlay_idx.reshape(-1).long(),
                               overlay_vals.detach().to(torch.float16))
    return t


def ceil_div(a, b):
    return (a + b - 1) // b


def lr_at(step, steps, lr_peak):
    """Warmup + cosine schedule of train.py:616-624."""
    warm = max(1, int(steps * 0.05))
    if step <= warm:
        return lr_peak * step / warm
    c = 0.5 * (1 + math.cos(math.pi * (step - warm) / (steps - warm)))
    return lr_peak / 10 + (lr_peak - lr_peak / 10) * c
