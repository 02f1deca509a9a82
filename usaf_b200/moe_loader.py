"""Device-resident expert store and gradient-capture stores.

Drop-in counterparts of ``usaf.moe_loader`` (usaf/moe_loader.py:60-631):

* ``QuantizedExpertCache``: holds the q4 dict in HBM (B200 fits every layer's
  int4 experts) as :class:`~usaf_b200.engine.Projection` objects; ``overlays``
  maps a parameter name to ``(active_idx, master)`` like the reference, and
  ``sync_resident`` pushes updated masters into the GEMM overlay.  The
  reference's LRU / prefetch / host streaming exists for 12 GB GPUs and has
  no counterpart here.
* ``SparseGradStore(active_idx, shapes)``: compact fp32 gradients aligned
  with ``active_idx``, written by the fused backward (SDDMM) in HBM.
* ``TopKImportanceStore(shapes, frac, cand_mult=2.0)``: per-expert top
  ``max(1, int(numel_e*frac*cand_mult))`` |grad| candidates, ``select(frac)``
  takes the per-tensor top ``int(numel*frac)`` of their union.

Both stores also accept the reference's ``add(full_name, ei, grad)`` call
with a CUDA tensor.  Ties in |grad| are broken by ascending flat index
(torch.topk leaves that order unspecified).
"""
from __future__ import annotations

from typing import Any, Dict, Optional, Tuple

import torch

from . import engine
from .engine import Projection


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


class SparseGradStore:
    def __init__(self, active_idx: Dict[str, torch.Tensor], shapes: Dict[str, Any],
                 device=None):
        self.compact: Dict[str, torch.Tensor] = {}
        self.active_idx: Dict[str, torch.Tensor] = {}
        self.shapes = dict(shapes)
        self._local: Dict[Tuple[str, int], Tuple[torch.Tensor, torch.Tensor]] = {}
        for name, idx in active_idx.items():
            dev = device if device is not None else (idx.device if idx.is_cuda else "cuda")
            idx = idx.reshape(-1).to(device=dev, dtype=torch.long)
            self.active_idx[name] = idx
            self.compact[name] = torch.zeros(idx.numel(), dtype=torch.float32, device=dev)

    def zero_(self) -> None:
        for v in self.compact.values():
            v.zero_()

    def add(self, full_name: str, ei: int, g: torch.Tensor) -> None:
        """Reference protocol (usaf/moe_loader.py:564-578): gather a dense
        per-expert gradient at the active coordinates of expert ``ei``."""
        if full_name not in self.compact:
            return
        if not g.is_cuda:
            raise TypeError("usaf_b200 stores take CUDA gradients")
        slice_size = _numel(self.shapes[full_name][1:])
        if g.numel() != slice_size:
            raise ValueError(f"{full_name}: expert gradient of {g.numel()} elements, expected {slice_size}")
        key = (full_name, int(ei))
        if key not in self._local:
            idx = self.active_idx[full_name]
            pos = ((idx // slice_size) == ei).nonzero().reshape(-1)
            self._local[key] = (idx[pos] - ei * slice_size, pos)
        local, pos = self._local[key]
        if pos.numel():
            self.compact[full_name].index_add_(0, pos, g.detach().reshape(-1).gather(0, local).float())

    def n_captured(self) -> int:
        return len(self.compact)


class TopKImportanceStore:
    def __init__(self, shapes: Dict[str, Any], frac: float, cand_mult: float = 2.0):
        self._shapes = dict(shapes)
        self._frac = frac
        self._cand = cand_mult
        self._vals: Dict[str, Dict[int, torch.Tensor]] = {n: {} for n in shapes}
        self._idx: Dict[str, Dict[int, torch.Tensor]] = {n: {} for n in shapes}

    def zero_(self) -> None:
        for n in self._vals:
            self._vals[n].clear()
            self._idx[n].clear()

    def _k_of(self, numel_e: int) -> int:
        return max(1, int(numel_e * self._frac * self._cand))

    def add(self, full_name: str, ei: int, g: torch.Tensor) -> None:
        """Reference protocol (usaf/moe_loader.py:604-611) for one expert."""
        if full_name not in self._vals:
            return
        if not g.is_cuda:
            raise TypeError("usaf_b200 stores take CUDA gradients")
        flat = g.detach().float().reshape(-1).abs()
        if flat.numel() != _numel(self._shapes[full_name][1:]):
            raise ValueError(f"{full_name}: expert gradient of {flat.numel()} elements, expected "
                             f"{_numel(self._shapes[full_name][1:])}")
        k = min(self._k_of(flat.numel()), flat.numel())
        v, i = engine.topk_desc(flat, k, idx_base=int(ei) * flat.numel())
        self._vals[full_name][int(ei)] = v
        self._idx[full_name][int(ei)] = i

    def add_dense_abs(self, full_name: str, absg: torch.Tensor,
                      experts: Optional[torch.Tensor] = None, expert_offset: int = 0) -> None:
        """All experts at once from the fused backward: ``absg`` is |grad| as
        fp32 [E, R, C]; experts without routed tokens are skipped like the
        reference's sparse dispatch (no hook fires for them).  ``absg[e]``
        is expert ``e + expert_offset`` of the full tensor (an expert shard)."""
        if full_name not in self._vals:
            return
        E = absg.shape[0]
        numel_e = absg[0].numel()
        if numel_e != _numel(self._shapes[full_name][1:]):
            raise ValueError(f"{full_name}: |grad| slices of {numel_e} elements, expected "
                             f"{_numel(self._shapes[full_name][1:])}")
        k = min(self._k_of(numel_e), numel_e)
        hit = range(E) if experts is None else experts.tolist()
        for ei in hit:
            eg = int(ei) + expert_offset
            v, i = engine.topk_desc(absg[ei].reshape(-1), k, idx_base=eg * numel_e)
            self._vals[full_name][eg] = v
            self._idx[full_name][eg] = i

    def add_from(self, full_name: str, block, which: str, expert_offset: int = 0) -> None:
        """Candidates of one projection straight from a block's backward
        (``block``: an engine MoEBlock or an ExpertParallelMoE shard whose
        expert ``e`` is expert ``e + expert_offset`` of the full tensor).  bf16
        gradients take the fused path (no dense |grad| buffer), others the
        dense |grad| buffer of :meth:`add_dense_abs`; both keep the experts
        with routed tokens and resolve equal scores to the lowest index."""
        if full_name not in self._vals:
            return
        numel_e = _numel(self._shapes[full_name][1:])
        k = min(self._k_of(numel_e), numel_e)
        res = block.expert_candidates(which, k)
        if res is None:
            self.add_dense_abs(full_name, block.dense_abs_grad(which), block.hit_experts(), expert_offset)
            return
        vals, idx, experts = res
        base = expert_offset * numel_e
        for row, e in enumerate(experts.tolist()):
            eg = int(e) + expert_offset
            self._vals[full_name][eg] = vals[row * k:(row + 1) * k]
            self._idx[full_name][eg] = idx[row * k:(row + 1) * k] + base

    def candidates(self, name):
        """Per expert (scores, flat indices) in descending score order, equal
        scores by ascending index (torch.topk's sorted output)."""
        vals, idxs = {}, {}
        for e, v in self._vals[name].items():
            i = self._idx[name][e]
            if v.numel():
                vals[e], idxs[e] = engine.topk_desc(v, v.numel(), idx_map=i.to(torch.int64).contiguous())
            else:
                vals[e], idxs[e] = v, i
        return vals, idxs

    def select(self, frac: Optional[float] = None) -> Dict[str, torch.Tensor]:
        """Per-tensor top ``min(max(1,int(numel*frac)), n_cand)`` of the
        candidates (usaf/moe_loader.py:613-628), descending score."""
        frac = self._frac if frac is None else frac
        out: Dict[str, torch.Tensor] = {}
        for name, shape in self._shapes.items():
            if not self._vals[name]:
                continue
            vals, idxs = self.candidate_list(name)
            k = min(max(1, int(_numel(shape) * frac)), vals.numel())
            out[name] = select_candidates(vals, idxs, k)
        return out

    def candidate_list(self, name, device=None):
        """All candidates of one tensor (scores, flat indices), expert order."""
        keys = sorted(self._vals[name])
        if not keys:
            dev = device if device is not None else "cuda"
            return (torch.empty(0, dtype=torch.float32, device=dev),
                    torch.empty(0, dtype=torch.int64, device=dev))
        return (torch.cat([self._vals[name][e] for e in keys]),
                torch.cat([self._idx[name][e] for e in keys]))

    def n_captured(self) -> int:
        return sum(len(d) for d in self._vals.values())


class DenseAbsGradStore:
    """Full-size sums of |gradient| of int4 expert tensors, fp32 [E, R, C] on
    the device: the importance scores of usaf/importance.py:60-97 for experts
    whose gradients never exist as a parameter ``.grad`` here.  Filled through
    the ``_grad_capture`` protocol by the fused backward (every expert, zeros
    for experts without routed tokens)."""

    def __init__(self, shapes: Dict[str, Any]):
        self._shapes = dict(shapes)
        self.scores: Dict[str, torch.Tensor] = {}

    def zero_(self) -> None:
        self.scores.clear()

    def add_dense_abs(self, full_name: str, absg: torch.Tensor,
                      experts: Optional[torch.Tensor] = None, expert_offset: int = 0) -> None:
        if full_name not in self._shapes:
            return
        if not absg.is_cuda:
            raise TypeError("usaf_b200 stores take CUDA gradients")
        acc = self.scores.get(full_name)
        if acc is None:
            acc = torch.zeros(tuple(self._shapes[full_name]), dtype=torch.float32, device=absg.device)
            self.scores[full_name] = acc
        acc[expert_offset:expert_offset + absg.shape[0]].add_(absg)

    def n_captured(self) -> int:
        return len(self.scores)


def select_candidates(vals: torch.Tensor, idxs: torch.Tensor, k: int) -> torch.Tensor:
    """Flat indices of the top ``k`` candidate scores, descending score; equal
    scores resolve to the lowest flat index (candidates are ordered by index
    before the select)."""
    sk, perm = engine.sort_u32(idxs, torch.arange(idxs.numel(), device=idxs.device))
    _, sel = engine.topk_desc(vals[perm], k, idx_map=sk.to(torch.int64), want_vals=False)
    return sel


class QuantizedExpertCache:
    """int4 experts resident in HBM (usaf/moe_loader.py:60-524 without the
    host-RAM streaming machinery).

    ``quantized_dict`` maps ``"<module>.gate_up_proj"`` / ``".down_proj"`` to the
    reference's q4 entries (dict ``{"q","s","z","shape","group_size"}`` or
    4-tuple).  ``overlays[name] = (active_idx, master)`` installs trained
    coordinates; ``sync_resident`` refreshes their values after an optimizer
    step (the fused SparseAdam already does this when given the projection).
    """

    def __init__(self, quantized_dict: Dict[str, Any], device="cuda", max_cached: int = 0,
                 group_size: int = 128, dtype: torch.dtype = torch.bfloat16):
        self._device = torch.device(device)
        self._group_size = group_size
        self._dtype = dtype
        self.projections: Dict[str, Projection] = {}
        for name, entry in quantized_dict.items():
            if isinstance(entry, dict) and "q" in entry:
                q, s, z, shape = entry["q"], entry["s"], entry["z"], entry["shape"]
                gs = entry.get("group_size", group_size)
            elif isinstance(entry, tuple) and len(entry) == 4:
                (q, s, z, shape), gs = entry, group_size
            else:
                continue
            if len(shape) != 3:
                continue
            self.projections[name] = Projection(
                torch.as_tensor(q).to(self._device), torch.as_tensor(s).to(self._device),
                torch.as_tensor(z).to(self._device), shape, gs, dtype)
        self.overlays: Dict[str, Tuple[torch.Tensor, torch.Tensor]] = {}

    def projection(self, name: str) -> Projection:
        return self.projections[name]

    def apply_resident_overlays(self, active_idx, masters) -> None:
        for name, idx in active_idx.items():
            if name in self.projections:
                m = masters[name]
                m = m.data if isinstance(m, torch.nn.Parameter) else m
                self.projections[name].set_overlay(idx.to(self._device), m.to(self._device))
                self.overlays[name] = (idx, m)

    def sync_resident(self, active_idx, masters) -> None:
        for name in active_idx:
            if name in self.projections and self.projections[name].n_ov:
                m = masters[name]
                m = m.data if isinstance(m, torch.nn.Parameter) else m
                self.projections[name].update_overlay_values(m)

    def dequant(self, name: str) -> torch.Tensor:
        """fp16 dequant of the ORIGINAL int4 weights (no overlay)."""
        return self.projections[name].dequant(torch.float16)
