"""Qwen3-MoE block on the B200 kernels (drop-in for usaf/qwen3moe_dml.py).

``patch_qwen3moe_for_b200()`` replaces ``Qwen3MoeSparseMoeBlock.forward`` and
``Qwen3MoeExperts.forward`` of transformers' modeling_qwen3_moe, as
``patch_qwen3moe_for_dml()`` does (usaf/qwen3moe_dml.py:89-94).  The block
forward keeps the reference's semantics (usaf/qwen3moe_dml.py:67-86): router
logits in the activation dtype, fp32 softmax, threshold mask
``probs >= k-th largest`` (ties admit more than top_k experts), optional
renormalisation, weights in the activation dtype, and the expert combine
summed in fp32 in ascending expert order.

Expert weights are not read from the module's ``gate_up_proj`` /
``down_proj`` parameters (the reference fills those per forward from its
int4 cache, train.py:187-197); they come from an int4 store attached with
:func:`attach_int4_experts`, resident in HBM with the overlay of trained
coordinates.

Gradient capture keeps the reference protocol (usaf/qwen3moe_dml.py:10-19,
30-56): when ``experts._grad_capture = (store, prefix)`` is set, the backward
adds the expert-weight gradients to ``store`` under
``f"{prefix}.gate_up_proj"`` / ``f"{prefix}.down_proj"``:
:class:`usaf_b200.moe_loader.SparseGradStore` receives compact gradients at
its active coordinates (computed without forming the dense gradient),
:class:`usaf_b200.moe_loader.TopKImportanceStore` receives the dense
|gradient| of every routed expert, :class:`usaf_b200.moe_loader.DenseAbsGradStore`
sums it full-size (the importance scores).  Other store types raise ``TypeError``
(the dense CPU buffers of the reference's dict protocol are not produced).
The router weight receives its gradient through autograd.
"""
from __future__ import annotations

import contextlib
from typing import Dict, List, Optional, Tuple

import torch

from .engine import BackwardScratch, BlockDims, MoEBlock, Projection, pair_capacity
from .moe_loader import DenseAbsGradStore, SparseGradStore, TopKImportanceStore


def int4_projection(entry, shape, group_size: int = 128, dtype=torch.bfloat16,
                    device=None) -> Projection:
    """One q4 entry of the reference's store (a dict with ``q``, ``s``, ``z``
    or a ``(q, s, z, ...)`` tuple, train.py:175-177) as a device Projection."""
    if isinstance(entry, dict):
        q, s, z = entry["q"], entry["s"], entry["z"]
    else:
        q, s, z = entry[0], entry[1], entry[2]
    dev = torch.device(device) if device is not None else torch.device("cuda")
    return Projection(q.to(dev), s.to(dev), z.to(dev), shape, group_size, dtype)


def attach_int4_experts(experts: torch.nn.Module, gate_up: Projection, down: Projection,
                        expert_parallel: bool = False, group=None) -> None:
    """Give a ``Qwen3MoeExperts`` module its int4 expert weights.

    ``expert_parallel``: the experts are sharded over the torch.distributed
    ``group`` (None: the default group); this rank's ``gate_up`` / ``down``
    hold its E/W experts ([E/W, 2I, H] and [E/W, H, I]) and rank r owns
    experts [r E/W, (r+1) E/W).  Every rank routes its own tokens with the
    replicated router; the block exchanges rows with the experts' owners over
    NCCL, and the router gradient is summed over the ranks.  Captured
    gradients are those of this rank's experts under the full tensors'
    names and flat indices."""
    if gate_up.E != down.E or gate_up.C != down.R or gate_up.R != 2 * down.C:
        raise ValueError("gate_up [E,2I,H] and down [E,H,I] shapes do not match")
    experts._usaf_int4 = (gate_up, down)
    experts._usaf_ep = bool(expert_parallel)
    experts._usaf_ep_group = group


def _int4_of(experts) -> Tuple[Projection, Projection]:
    p = getattr(experts, "_usaf_int4", None)
    if p is None:
        raise RuntimeError("no int4 expert weights attached (usaf_b200.qwen3moe.attach_int4_experts)")
    return p


# Workspace policy of the patched blocks (configure_workspaces)
_POLICY = {"pair_factor": 2.0, "share_backward": False}
_SHARED: Dict[tuple, BackwardScratch] = {}


def configure_workspaces(pair_factor: float = 2.0, share_backward: bool = False) -> None:
    """How the patched blocks size their device workspaces (blocks created
    afterwards; a block keeps its workspace for its lifetime).

    Every block keeps what its backward needs from its forward (permuted
    tokens, gate/up, h, the routing plan: ~1.1 GB per C3 layer at 8192
    tokens and ``pair_factor`` 1.25).  ``share_backward`` lets all blocks of
    the same sizes share one set of their backward-only buffers (the
    backwards of a model run one after another), which is what makes a deep
    model fit: ~1 GB once instead of per layer.  ``pair_factor`` sizes the
    pair buffers at ``T * ceil(pair_factor * top_k)`` pairs: threshold ties
    add pairs, and a batch that exceeds the buffer is refused (the trainer
    raises ``UsafError`` on its next host read)."""
    if pair_factor < 1:
        raise ValueError("pair_factor must be >= 1")
    _POLICY["pair_factor"] = float(pair_factor)
    _POLICY["share_backward"] = bool(share_backward)


def _block_for(owner, T: int, H: int, E: int, I: int, top_k: int, norm: bool, dtype, device,
               pair_factor: Optional[float] = None) -> MoEBlock:
    """Workspace of one module for T tokens (kept between the forward and
    the backward; one per module, so layers do not share what the backward
    reads from the forward)."""
    pf = _POLICY["pair_factor"] if pair_factor is None else pair_factor
    cache: Dict[tuple, MoEBlock] = owner.__dict__.setdefault("_usaf_blocks", {})
    key = (T, top_k, pf, norm)
    blk = cache.get(key)
    if blk is None:
        dims = BlockDims(T, H, E, I, top_k, norm, dtype)
        scratch = None
        if _POLICY["share_backward"]:
            dev = torch.device(device)
            P_cap = pair_capacity(T, E, top_k, pf)
            skey = (P_cap, T, H, E, I, dtype, dev)
            scratch = _SHARED.get(skey)
            if scratch is None:
                scratch = _SHARED[skey] = BackwardScratch(P_cap, T, H, E, I, dtype, dev)
        blk = MoEBlock(dims, device, pf, scratch)
        cache[key] = blk
    return blk


def _ep_for(owner, T: int, w_r: torch.Tensor, top_k: int, norm: bool, gu: Projection,
            dn: Projection, group):
    """Expert-parallel workspace of one module for T tokens (one per module).

    The key holds everything the workspace is built from: the pair factor in
    force, and the projections themselves (re-attaching other int4 weights
    builds a new workspace instead of reusing one bound to the old ones; the
    cached workspace keeps its projections alive, so their ids stay unique)."""
    from .expert_parallel import ExpertParallelMoE
    cache = owner.__dict__.setdefault("_usaf_ep_moes", {})
    pf = _POLICY["pair_factor"]
    key = (T, top_k, norm, pf, id(gu), id(dn), id(group))
    moe = cache.get(key)
    if moe is None:
        moe = ExpertParallelMoE(w_r, gu, dn, top_k, T, norm, group, pf)
        cache[key] = moe
    return moe


def workspaces(model: torch.nn.Module) -> List[MoEBlock]:
    """Every block workspace the patched forwards created inside ``model``
    (the source-side block of each expert-parallel workspace included)."""
    out: List[MoEBlock] = []
    for m in model.modules():
        out.extend(m.__dict__.get("_usaf_blocks", {}).values())
        out.extend(ep.src for ep in m.__dict__.get("_usaf_ep_moes", {}).values())
    return out


def _capture(experts, blk: MoEBlock, gu: Projection, dn: Projection) -> None:
    cap = getattr(experts, "_grad_capture", None)
    if cap is None:
        return
    store, prefix = cap
    if isinstance(store, SparseGradStore):
        n_gu, n_dn = f"{prefix}.gate_up_proj", f"{prefix}.down_proj"
        for n, p in ((n_gu, gu), (n_dn, dn)):
            if n in store.compact and p.n_ov != store.compact[n].numel():
                raise ValueError(f"{n}: overlay and store hold different active sets")
        empty = torch.empty(0, device=blk.device)
        gu_s = gu if n_gu in store.compact else _NoOverlay()
        dn_s = dn if n_dn in store.compact else _NoOverlay()
        blk.sparse_grads(gu_s, dn_s, store.compact.get(n_gu, empty), store.compact.get(n_dn, empty))
    elif isinstance(store, TopKImportanceStore):
        for which in ("gate_up_proj", "down_proj"):
            store.add_from(f"{prefix}.{which}", blk, which)
    elif isinstance(store, DenseAbsGradStore):
        for which in ("gate_up_proj", "down_proj"):
            store.add_dense_abs(f"{prefix}.{which}", blk.dense_abs_grad(which))
    else:
        raise TypeError("usaf_b200 captures into SparseGradStore / TopKImportanceStore / "
                        f"DenseAbsGradStore, not {type(store).__name__}")


class _NoOverlay:
    """Stands in for a projection whose gradient the store does not want."""
    n_ov = 0


class _BlockFn(torch.autograd.Function):
    """Router + experts of one block; saves the routing plan in the module's
    workspace for the backward."""

    @staticmethod
    def forward(ctx, hs, w_r, block):
        gate, experts = block.gate, block.experts
        gu, dn = _int4_of(experts)
        T, H = hs.shape
        blk = _block_for(block, T, H, w_r.shape[0], dn.C, gate.top_k, bool(gate.norm_topk_prob),
                         hs.dtype, hs.device)
        y = blk.forward(hs, w_r, gu, dn).clone()
        ctx.block, ctx.blk = block, blk
        ctx.save_for_backward(hs, w_r)
        return y

    @staticmethod
    def backward(ctx, dy):
        hs, w_r = ctx.saved_tensors
        blk, block = ctx.blk, ctx.block
        gu, dn = _int4_of(block.experts)
        dx, dw_r = blk.backward(dy.contiguous(), hs, w_r, gu, dn)
        _capture(block.experts, blk, gu, dn)
        return dx.clone(), (dw_r.clone() if ctx.needs_input_grad[1] else None), None


class _EPBlockFn(torch.autograd.Function):
    """Router + experts of one block with the experts sharded over ranks
    (``attach_int4_experts(..., expert_parallel=True)``)."""

    @staticmethod
    def forward(ctx, hs, w_r, block):
        experts = block.experts
        gu, dn = _int4_of(experts)
        moe = _ep_for(block, hs.shape[0], w_r, block.gate.top_k, bool(block.gate.norm_topk_prob),
                      gu, dn, experts._usaf_ep_group)
        y = moe.forward(hs, w_r).clone()
        ctx.block, ctx.moe = block, moe
        ctx.save_for_backward(hs, w_r)
        return y

    @staticmethod
    def backward(ctx, dy):
        hs, w_r = ctx.saved_tensors
        moe, experts = ctx.moe, ctx.block.experts
        cap = getattr(experts, "_grad_capture", None)
        cg = cd = None
        if cap is not None and isinstance(cap[0], SparseGradStore):
            store, prefix = cap
            gu, dn = _int4_of(experts)
            cg = store.compact.get(f"{prefix}.gate_up_proj")
            cd = store.compact.get(f"{prefix}.down_proj")
            for c, p, nm in ((cg, gu, "gate_up_proj"), (cd, dn, "down_proj")):
                if c is not None and p.n_ov != c.numel():
                    raise ValueError(f"{prefix}.{nm}: overlay and store hold different active sets")
            if cg is None or cd is None:   # the store wants one projection: the other's grads are discarded
                cg = cg if cg is not None else torch.zeros(gu.n_ov, device=hs.device)
                cd = cd if cd is not None else torch.zeros(dn.n_ov, device=hs.device)
        dx, dw_r = moe.backward(dy.contiguous(), hs, w_r, reduce_router=True, compact_gu=cg,
                                compact_dn=cd)
        if cap is not None and not isinstance(cap[0], SparseGradStore):
            _capture_ep(experts, moe, cap)
        return dx.clone(), (dw_r.clone() if ctx.needs_input_grad[1] else None), None


def _capture_ep(experts, moe, cap) -> None:
    """Importance captures of this rank's experts, numbered as experts of the
    full tensors (``expert_offset``); the per-tensor selection over all ranks
    is the caller's (``expert_parallel.global_select``)."""
    store, prefix = cap
    e0 = moe.rank * moe.El
    if isinstance(store, TopKImportanceStore):
        for which in ("gate_up_proj", "down_proj"):
            store.add_from(f"{prefix}.{which}", moe, which, expert_offset=e0)
    elif isinstance(store, DenseAbsGradStore):
        for which in ("gate_up_proj", "down_proj"):
            store.add_dense_abs(f"{prefix}.{which}", moe.dense_abs_grad(which), expert_offset=e0)
    else:
        raise TypeError("usaf_b200 captures into SparseGradStore / TopKImportanceStore / "
                        f"DenseAbsGradStore, not {type(store).__name__}")


class _ExpertsFn(torch.autograd.Function):
    """Experts with caller-given dense weights (the reference's
    ``experts(hidden_states, weights)`` call)."""

    @staticmethod
    def forward(ctx, hs, weights, experts):
        gu, dn = _int4_of(experts)
        T, H = hs.shape
        # pairs per token, rounded up: the workspace must hold every nonzero weight
        kmax = max(1, -(-int((weights != 0).sum().item()) // max(T, 1)))
        blk = _block_for(experts, T, H, weights.shape[1], dn.C, kmax, False, hs.dtype, hs.device,
                         pair_factor=1)
        y = blk.experts_forward(hs, weights.contiguous(), gu, dn).clone()
        ctx.experts, ctx.blk = experts, blk
        return y

    @staticmethod
    def backward(ctx, dy):
        blk, experts = ctx.blk, ctx.experts
        gu, dn = _int4_of(experts)
        dx, dwts = blk.experts_backward(dy.contiguous(), gu, dn)
        _capture(experts, blk, gu, dn)
        return dx.clone(), (dwts if ctx.needs_input_grad[1] else None), None


def b200_qwen3_moe_block_forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
    """``dml_qwen3_moe_block_forward`` (usaf/qwen3moe_dml.py:67-86) on B200."""
    batch_size, sequence_length, hidden_dim = hidden_states.shape
    hs = hidden_states.reshape(-1, hidden_dim).contiguous()
    fn = _EPBlockFn if getattr(self.experts, "_usaf_ep", False) else _BlockFn
    y = fn.apply(hs, self.gate.weight, self)
    return y.view(batch_size, sequence_length, hidden_dim)


def b200_qwen3_experts_forward(self, hidden_states: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """``dml_qwen3_experts_forward`` (usaf/qwen3moe_dml.py:24-64) on B200:
    ``weights`` is the dense [T, E] routing matrix (zeros off-route).  Only
    routed (nonzero) entries are computed, so the gradient of ``weights`` is
    ``dy[t] . y_e[t]`` at routed entries and 0 elsewhere; the reference's
    dense-masked loop also fills the off-route entries, which its block
    discards through the routing mask."""
    if getattr(self, "_usaf_ep", False):
        raise NotImplementedError("expert-parallel experts run through the block forward "
                                  "(Qwen3MoeSparseMoeBlock), which routes and exchanges the tokens")
    return _ExpertsFn.apply(hidden_states.contiguous(), weights, self)


def patch_qwen3moe_for_b200():
    """Install the B200 forwards (affects all model instances), like
    ``patch_qwen3moe_for_dml`` (usaf/qwen3moe_dml.py:89-94)."""
    from transformers.models.qwen3_moe import modeling_qwen3_moe
    modeling_qwen3_moe.Qwen3MoeExperts.forward = b200_qwen3_experts_forward
    modeling_qwen3_moe.Qwen3MoeSparseMoeBlock.forward = b200_qwen3_moe_block_forward
    return modeling_qwen3_moe


@contextlib.contextmanager
def without_dense_experts():
    """Build ``Qwen3MoeExperts`` modules without their dense weight tensors.

    The patched forwards read the int4 store attached with
    :func:`attach_int4_experts`, never ``gate_up_proj`` / ``down_proj`` (the
    reference fills those per forward from its cache, train.py:187-197).
    Inside this context a new experts module gets both as empty parameters
    on the current default device: a 48-layer C3 model would otherwise
    allocate 116 GB of fp32 expert weights before they could be quantized."""
    from transformers.models.qwen3_moe import modeling_qwen3_moe as mq
    orig = mq.Qwen3MoeExperts.__init__

    def init(self, config):
        with torch.device("meta"):
            orig(self, config)
        self.gate_up_proj = torch.nn.Parameter(torch.empty(0), requires_grad=False)
        self.down_proj = torch.nn.Parameter(torch.empty(0), requires_grad=False)

    mq.Qwen3MoeExperts.__init__ = init
    try:
        yield
    finally:
        mq.Qwen3MoeExperts.__init__ = orig
