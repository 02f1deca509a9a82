"""Expert parallelism over NCCL: experts sharded across the ranks of one box.

Rank r of W owns experts [r*El, (r+1)*El) (El = E/W): their int4 weights,
overlays, masters, Adam moments and compact gradients live only there, so
SparseAdam is rank-local.  Tokens stay data-parallel: each rank routes its
own batch with the replicated router (routing does not depend on W), builds
its expert-major ``x_perm`` over all E experts, and one all-to-all per
direction moves the rows to the experts' owners and the results back.  The
router gradient is summed over ranks (all-reduce).  The reference runs in a
single process; the row order on an owner (per expert: source rank, then the
source's slot order) equals the slot order of one process holding the
concatenated batches, so an expert sees its tokens in the same order either
way.

Kernels never read another GPU's memory: NCCL delivers every row into a
local buffer first.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Dict, List, Optional

import torch
import torch.distributed as dist

from . import _lib
from ._lib import call, ptr, stream
from .engine import BlockDims, MoEBlock, Projection, _check_act, _map, expert_candidates
from .moe_loader import SparseGradStore, TopKImportanceStore, select_candidates
from .sparse_optim import SparseAdam


@dataclass
class ExchangePlan:
    send_splits: List[int]       # rows this rank sends to each rank
    recv_splits: List[int]       # rows this rank receives from each rank
    recv_counts: torch.Tensor    # [W, El] int32: rows from source s for local expert e

    @property
    def n_send(self) -> int:
        return sum(self.send_splits)

    @property
    def n_recv(self) -> int:
        return sum(self.recv_splits)


def device_permute(counts: torch.Tensor, rows_in: torch.Tensor, rows_out: torch.Tensor,
                   inverse: bool, err: torch.Tensor) -> None:
    """(source, expert) block order <-> (expert, source) on the device."""
    W, El = counts.shape
    n = rows_in.shape[0]
    call("usaf_ep_permute", ptr(counts), W, El, n, ptr(rows_in), ptr(rows_out),
         rows_in[0].numel() * rows_in.element_size() if n else 16, int(inverse), ptr(err), stream())


class ExpertExchange:
    """Moves routed rows between the ranks of an expert-parallel group.

    ``permute`` regroups received rows (default: the device kernel); the
    all-to-alls go through ``torch.distributed`` (NCCL on GPUs)."""

    def __init__(self, num_experts: int, group=None,
                 permute: Optional[Callable] = None, err: Optional[torch.Tensor] = None):
        self.group = group
        self.W = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.W:
            raise ValueError(f"{num_experts} experts do not split over {self.W} ranks")
        self.E = num_experts
        self.El = num_experts // self.W
        self._permute = permute or device_permute
        self.err = err
        self._bufs: Dict[tuple, torch.Tensor] = {}

    def _buf(self, tag, rows: int, like: torch.Tensor) -> torch.Tensor:
        key = (tag, like.dtype, like.shape[1:], like.device)
        b = self._bufs.get(key)
        if b is None or b.shape[0] < rows:
            b = torch.empty((max(rows, 1),) + tuple(like.shape[1:]), dtype=like.dtype, device=like.device)
            self._bufs[key] = b
        return b

    def plan(self, expert_cnt: torch.Tensor) -> ExchangePlan:
        """Exchange per-expert row counts (int32 [E], this rank's dispatch)."""
        send = expert_cnt[: self.E].reshape(self.W, self.El).contiguous()
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        both = torch.stack([send.sum(1), recv.sum(1)]).cpu()   # the one host sync
        return ExchangePlan(both[0].tolist(), both[1].tolist(), recv)

    def to_owners(self, rows_src: torch.Tensor, xp: ExchangePlan, out: torch.Tensor) -> None:
        """rows_src: this rank's expert-major rows [>= n_send, ...];
        out: expert-major rows of the local experts [>= n_recv, ...]."""
        buf = self._buf("recv", xp.n_recv, rows_src)
        dist.all_to_all_single(buf[: xp.n_recv], rows_src[: xp.n_send], xp.recv_splits,
                               xp.send_splits, group=self.group)
        if xp.n_recv:
            self._permute(xp.recv_counts, buf[: xp.n_recv], out[: xp.n_recv], False, self.err)

    def to_sources(self, rows_own: torch.Tensor, xp: ExchangePlan, out: torch.Tensor,
                   async_op: bool = False):
        """Inverse of :meth:`to_owners`: rows_own (expert-major, local experts)
        go back to the ranks and slots they came from.  With ``async_op`` the
        all-to-all is left in flight (returns its work handle): kernels
        launched meanwhile overlap it, ``wait()`` orders the stream after it."""
        buf = self._buf("back", xp.n_recv, rows_own)
        if xp.n_recv:
            self._permute(xp.recv_counts, rows_own[: xp.n_recv], buf[: xp.n_recv], True, self.err)
        return dist.all_to_all_single(out[: xp.n_send], buf[: xp.n_recv], xp.send_splits,
                                      xp.recv_splits, group=self.group, async_op=async_op)

    def to_owners_start(self, rows_src: torch.Tensor, xp: ExchangePlan):
        """First half of :meth:`to_owners`: the all-to-all, left in flight."""
        buf = self._buf("recv", xp.n_recv, rows_src)
        work = dist.all_to_all_single(buf[: xp.n_recv], rows_src[: xp.n_send], xp.recv_splits,
                                      xp.send_splits, group=self.group, async_op=True)
        return work, buf

    def to_owners_finish(self, work, buf: torch.Tensor, xp: ExchangePlan, out: torch.Tensor) -> None:
        work.wait()
        if xp.n_recv:
            self._permute(xp.recv_counts, buf[: xp.n_recv], out[: xp.n_recv], False, self.err)


class ExpertParallelMoE:
    """One MoE layer, experts sharded over the group (forward, backward,
    sparse expert gradients).

    ``gu_local`` / ``dn_local`` hold this rank's El experts ([El, 2I, H] and
    [El, H, I]); ``w_r`` is the full replicated router [E, H]."""

    def __init__(self, w_r: torch.Tensor, gu_local: Projection, dn_local: Projection, top_k: int,
                 T: int, norm_topk_prob: bool = True, group=None, pair_factor: int = 2):
        E, H = w_r.shape
        self.dev = w_r.device
        self.dt = w_r.dtype
        self.dtc = _lib.dtype_code(w_r.dtype)
        self.gu, self.dn = gu_local, dn_local
        I = dn_local.C
        # source side: router, dispatch over all E experts, combine
        self.src = MoEBlock(BlockDims(T, H, E, I, top_k, norm_topk_prob, w_r.dtype), self.dev,
                            pair_factor)
        self.x_ = ExpertExchange(E, group, err=self.src.err)
        self.W, self.rank, self.El = self.x_.W, self.x_.rank, self.x_.El
        if gu_local.E != self.El or dn_local.E != self.El:
            raise ValueError(f"rank {self.rank} must hold {self.El} experts")
        self.H, self.I, self.E = H, I, E
        i32 = dict(dtype=torch.int32, device=self.dev)
        self.own_cnt = torch.zeros(self.El, **i32)
        self.own_off = torch.zeros(self.El + 1, **i32)
        self.own_n = torch.zeros(1, **i32)
        self.own_sched = torch.zeros(16, **i32)   # GEMM work counters of the owner plan
        self.cap = 0
        self.own = _lib.RoutePlan()
        self.xp: Optional[ExchangePlan] = None

    # owner-side buffers grow to the largest batch seen
    def _own_buffers(self, rows: int):
        if rows <= self.cap:
            return
        # grow with headroom: the routed rows drift up as the router trains, and every
        # regrowth allocates seven buffers (an allocation stalls the stream)
        cap = max(-(-int(rows * 1.25) // 256) * 256, 256)
        act = dict(dtype=self.dt, device=self.dev)
        H, I = self.H, self.I
        self.x_own = torch.empty(cap, H, **act)
        self.gu_own = torch.empty(cap, 2 * I, **act)
        self.h_own = torch.empty(cap, I, **act)
        self.y_own = torch.empty(cap, H, **act)
        self.dcur_own = torch.empty(cap, H, **act)
        self.dgu_own = torch.empty(cap, 2 * I, **act)
        self.dx_own = torch.empty(cap, H, **act)
        self.cap = cap
        p = self.own
        p.T, p.E, p.P_cap = 0, self.El, cap
        p.expert_cnt, p.expert_off, p.n_pairs = ptr(self.own_cnt), ptr(self.own_off), ptr(self.own_n)
        p.err = ptr(self.src.err)
        p.sched = ptr(self.own_sched)

    # ---------------------------------------------------------------- fwd ---
    def forward(self, x: torch.Tensor, w_r: torch.Tensor) -> torch.Tensor:
        s, d = self.src, self.src.d
        _check_act("x", x, (d.T, d.H), self.dt)
        _check_act("w_r", w_r, (d.E, d.H), self.dt)
        st = stream()
        call("usaf_router_fwd", ptr(x), ptr(w_r), self.dtc, d.T, d.H, d.E, d.top_k,
             int(d.norm_topk_prob), ptr(s.logits), ptr(s.probs), ptr(s.wsum), ptr(s.weights),
             ptr(s.router_ws), ptr(s.err), st)
        call("usaf_dispatch", s.plan, ptr(s.weights), ptr(x), self.dtc, d.H, ptr(s.x_perm), st)
        xp = self.x_.plan(s.expert_cnt)
        self.xp = xp
        self._own_buffers(xp.n_recv)
        call("usaf_ep_owner_counts", ptr(xp.recv_counts), self.W, self.El, ptr(self.own_cnt),
             ptr(self.own_off), ptr(self.own_n), st)
        self.x_.to_owners(s.x_perm, xp, self.x_own)
        call("usaf_expert_gate_up_fwd", self.own, self.gu.struct(), ptr(self.x_own), self.dtc,
             ptr(self.gu_own), ptr(self.h_own), st)
        call("usaf_expert_down_fwd", self.own, self.dn.struct(), ptr(self.h_own), self.dtc,
             ptr(self.y_own), st)
        self.x_.to_sources(self.y_own, xp, s.y_seg)
        call("usaf_combine", s.plan, ptr(s.y_seg), self.dtc, d.H, ptr(s.y), st)
        return s.y

    # ---------------------------------------------------------------- bwd ---
    def backward(self, dy: torch.Tensor, x: torch.Tensor, w_r: torch.Tensor,
                 reduce_router: bool = True, compact_gu: Optional[torch.Tensor] = None,
                 compact_dn: Optional[torch.Tensor] = None):
        """dX and the router gradient.  Given compact gradient vectors, the
        expert-weight gradients (:meth:`sparse_grads`) are computed while the
        dX rows travel back, and the router backward runs while the output
        gradients travel to the owners."""
        s, d, xp = self.src, self.src.d, self.xp
        _check_act("dy", dy, (d.T, d.H), self.dt)
        _check_act("x", x, (d.T, d.H), self.dt)
        _check_act("w_r", w_r, (d.E, d.H), self.dt)
        st = stream()
        call("usaf_combine_bwd", s.plan, ptr(dy), ptr(s.y_seg), self.dtc, d.H, ptr(s.dcur),
             ptr(s.dw_pair), st)
        work, buf = self.x_.to_owners_start(s.dcur, xp)
        call("usaf_router_bwd", s.plan, ptr(x), ptr(w_r), self.dtc, d.H, int(d.norm_topk_prob),
             ptr(s.probs), ptr(s.wsum), ptr(s.weights), ptr(s.dw_pair), ptr(s.dlogits),
             ptr(s.dw_r), ptr(s.dx_acc), ptr(s.router_ws), st)
        self.x_.to_owners_finish(work, buf, xp, self.dcur_own)
        call("usaf_expert_down_bwd", self.own, self.dn.struct(), ptr(self.dcur_own), ptr(self.gu_own),
             self.dtc, ptr(self.dgu_own), st)
        call("usaf_expert_gate_up_bwd", self.own, self.gu.struct(), ptr(self.dgu_own), self.dtc,
             ptr(self.dx_own), st)
        work = self.x_.to_sources(self.dx_own, xp, s.dx_seg, async_op=True)
        if compact_gu is not None and compact_dn is not None:
            self.sparse_grads(compact_gu, compact_dn)
        work.wait()
        call("usaf_gather_dx", s.plan, ptr(s.dx_seg), ptr(s.dx_acc), self.dtc, d.H, ptr(s.dx), st)
        dw_r = s.dw_r
        if reduce_router and self.W > 1:
            acc = s.dw_r.float()
            dist.all_reduce(acc, group=self.x_.group)
            dw_r = acc.to(self.dt)
        return s.dx, dw_r

    # ------------------------------------------------- expert weight grads ---
    def sparse_grads(self, compact_gu: torch.Tensor, compact_dn: torch.Tensor, scale: float = 1.0):
        """Compact gradients of this rank's experts (all ranks' tokens)."""
        st = stream()
        if self.gu.n_ov:
            call("usaf_sparse_dw", self.own, self.gu.struct(), ptr(self.dgu_own), ptr(self.x_own),
                 self.dtc, _map(self.gu), scale, ptr(compact_gu), ptr(self.gu.scratch), st)
        if self.dn.n_ov:
            call("usaf_sparse_dw", self.own, self.dn.struct(), ptr(self.dcur_own), ptr(self.h_own),
                 self.dtc, _map(self.dn), scale, ptr(compact_dn), ptr(self.dn.scratch), st)

    def hit_experts(self) -> torch.Tensor:
        """This rank's experts that received slots from any rank."""
        return (self.own_cnt > 0).nonzero().reshape(-1)

    def expert_candidates(self, which: str, k: int):
        """Per-expert top-``k`` |dW| candidates of this rank's experts (all
        ranks' tokens) without the dense buffer; None if not covered."""
        if which == "gate_up_proj":
            R, C, gout, gin = 2 * self.I, self.H, self.dgu_own, self.x_own
        else:
            R, C, gout, gin = self.H, self.I, self.dcur_own, self.h_own
        return expert_candidates(self.own, self.own_cnt, R, C, gout, gin, self.dtc, k)

    def dense_abs_grad(self, which: str) -> torch.Tensor:
        """|dW| of this rank's experts (fp32 [El, R, C]) for the importance pass."""
        if which == "gate_up_proj":
            R, C, gout, gin = 2 * self.I, self.H, self.dgu_own, self.x_own
        else:
            R, C, gout, gin = self.H, self.I, self.dcur_own, self.h_own
        out = torch.empty(self.El, R, C, dtype=torch.float32, device=self.dev)
        call("usaf_expert_dense_dw", self.own, R, C, ptr(gout), ptr(gin), self.dtc, ptr(out), stream())
        return out

    def check(self):
        self.src.check()

    def n_rows_host(self) -> int:
        """Rows this rank's experts processed in the last forward."""
        return int(self.own_n.item())


def global_select(cand_vals: torch.Tensor, cand_idx: torch.Tensor, k: int, group=None) -> torch.Tensor:
    """Top-k over the union of every rank's candidates of one tensor (the
    per-tensor select of usaf/moe_loader.py:613-628 across the expert
    shards); every rank gets the same global flat indices, equal to the
    single-process selection over the same candidates."""
    W = dist.get_world_size(group)
    n = torch.tensor([cand_vals.numel()], device=cand_vals.device, dtype=torch.int64)
    ns = [torch.zeros_like(n) for _ in range(W)]
    dist.all_gather(ns, n, group=group)
    ns = [int(v.item()) for v in ns]
    m = max(max(ns), 1)
    pv = torch.zeros(m, device=cand_vals.device, dtype=torch.float32)
    pi = torch.zeros(m, dtype=torch.int64, device=cand_vals.device)
    pv[: cand_vals.numel()] = cand_vals
    pi[: cand_idx.numel()] = cand_idx
    gv = [torch.empty_like(pv) for _ in range(W)]
    gi = [torch.empty_like(pi) for _ in range(W)]
    dist.all_gather(gv, pv, group=group)
    dist.all_gather(gi, pi, group=group)
    vals = torch.cat([g[:c] for g, c in zip(gv, ns)])
    idx = torch.cat([g[:c] for g, c in zip(gi, ns)])
    return select_candidates(vals, idx, min(k, vals.numel()))


class ExpertParallelLayer:
    """The sparse training step of one MoE layer over an expert shard
    (the expert-parallel counterpart of :class:`usaf_b200.layer.SparseMoELayer`).

    Parameter names and flat indices are those of the full [E, R, C] tensors;
    this rank stores and updates only the coordinates of its own experts."""

    def __init__(self, w_r: torch.Tensor, gu_local: Projection, dn_local: Projection, top_k: int,
                 T: int, norm_topk_prob: bool = True, prefix: str = "layer.mlp.experts", group=None):
        self.moe = ExpertParallelMoE(w_r, gu_local, dn_local, top_k, T, norm_topk_prob, group)
        self.group = group
        self.w_r = w_r
        self.prefix = prefix
        m = self.moe
        self.e0 = m.rank * m.El
        self.names = {f"{prefix}.gate_up_proj": gu_local, f"{prefix}.down_proj": dn_local}
        self.which = {f"{prefix}.gate_up_proj": "gate_up_proj", f"{prefix}.down_proj": "down_proj"}
        self.full_shapes = {n: (m.E,) + tuple(p.shape[1:]) for n, p in self.names.items()}
        self.local_shapes = {n: p.shape for n, p in self.names.items()}

    def _numel_e(self, name):
        p = self.names[name]
        return p.R * p.C

    def importance(self, x, dy, frac: float, cand_mult: float = 2.0) -> Dict[str, torch.Tensor]:
        """Dense |grad| pass and the global per-tensor top-k selection
        (usaf/moe_loader.py:604-628 over all shards); returns this rank's
        selected coordinates as flat indices of its local [El, R, C] tensors,
        in the global descending-score order."""
        m = self.moe
        m.forward(x, self.w_r)
        m.backward(dy, x, self.w_r, reduce_router=False)
        store = TopKImportanceStore(self.full_shapes, frac, cand_mult)
        for name in self.names:
            store.add_from(name, m, self.which[name], expert_offset=self.e0)
        out = {}
        for name, shape in self.full_shapes.items():
            vals, idxs = store.candidate_list(name, device=m.dev)
            numel = shape[0] * shape[1] * shape[2]
            g = global_select(vals, idxs, max(1, int(numel * frac)), self.group)
            ne = self._numel_e(name)
            lo, hi = self.e0 * ne, (self.e0 + m.El) * ne
            out[name] = g[(g >= lo) & (g < hi)] - lo
        return out

    def init_selection(self, active_local: Dict[str, torch.Tensor], lr=1e-4, weight_decay=0.01,
                       router_lr=None):
        self.active = {n: a.reshape(-1).long() for n, a in active_local.items()}
        for name, p in self.names.items():   # compact vectors in CSR order (identity maps)
            if name in self.active:
                self.active[name] = self.active[name][p.csr_order(self.active[name])]
        self.masters = {}
        for name, p in self.names.items():
            deq = p.dequant(torch.float16).reshape(-1)
            self.masters[name] = deq.index_select(0, self.active[name]).float()
            p.set_overlay(self.active[name], self.masters[name])
        self.store = SparseGradStore(self.active, self.local_shapes)
        params = {n: torch.nn.Parameter(v, requires_grad=False) for n, v in self.masters.items()}
        self.opt = SparseAdam(params, active_idx=self.active, lr=lr, weight_decay=weight_decay,
                              compact_params=True)
        for name, p in self.names.items():
            self.opt.bind_projection(name, p)
        self.params = params
        E, H = self.w_r.shape
        rname = self.prefix.replace(".experts", ".gate.weight")
        self.router_param = torch.nn.Parameter(self.w_r, requires_grad=False)
        self.router_opt = SparseAdam({rname: self.router_param},
                                     active_idx={rname: torch.arange(E * H, device=self.w_r.device)},
                                     lr=router_lr if router_lr is not None else lr,
                                     weight_decay=weight_decay)

    def train_step(self, x, dy, loss_scale: float = 1.0):
        """Forward, backward (router gradient summed over ranks), expert
        gradients of the local shard, SparseAdam on the shard and the router."""
        m = self.moe
        self.store.zero_()
        y = m.forward(x, self.w_r)
        n_gu, n_dn = list(self.names)
        dx, dw_r = m.backward(dy, x, self.w_r, compact_gu=self.store.compact[n_gu],
                              compact_dn=self.store.compact[n_dn])
        self.opt.step(compact_grads=self.store.compact, grad_div=float(loss_scale))
        self.router_param.grad = dw_r
        self.router_opt.step(grad_div=float(loss_scale))
        self.router_param.grad = None
        return y, dx, dw_r
