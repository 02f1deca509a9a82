"""Device-resident engine of the MoE expert hot path.

``Projection`` holds one int4 expert tensor (``gate_up_proj [E,2I,H]`` or
``down_proj [E,H,I]`` in the usaf.quantization layout) and the overlay of its
trained coordinates.  ``MoEBlock`` owns the per-step workspace and sequences
the C-ABI kernels for one forward/backward of the block:

  forward : router -> dispatch -> gate_up GEMM + SwiGLU -> down GEMM -> combine
  backward: combine bwd -> router bwd -> down dX GEMM + SwiGLU bwd
            -> gate_up dX GEMM -> dX gather; expert grads at the selected
            coordinates (SDDMM) or dense |grad| for importance.

Reference: usaf/qwen3moe_dml.py:24-86 (block), benchmarks/kaggle_t4_bench.py:
284-328 (dispatch), usaf/moe_loader.py:226-247, 425-443, 527-631 (weights,
overlays, stores).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib
from ._lib import call, ptr, stream


def _i32(t):
    return t.to(torch.int32).contiguous()


def sort_u32(keys: torch.Tensor, payload: torch.Tensor, descending: bool = False):
    """Stable device radix sort of int32/uint32 keys (< 2^31 here) with int64 payload."""
    n = keys.numel()
    kin = _i32(keys)
    vin = payload.to(torch.int64).contiguous()
    kout = torch.empty_like(kin)
    vout = torch.empty_like(vin)
    if n == 0:
        return kout, vout
    scratch = torch.empty(int(_lib.LIB.usaf_sort_scratch_bytes(n)), dtype=torch.uint8,
                          device=keys.device)
    call("usaf_sort_u32", ptr(kin), ptr(vin), n, ptr(kout), ptr(vout), int(descending),
         ptr(scratch), stream())
    return kout, vout


def expert_candidates(plan, expert_cnt: torch.Tensor, R: int, C: int, gout: torch.Tensor,
                      gin: torch.Tensor, dtc: int, k: int):
    """Per-expert top ``k`` of |grad_e| (TopKImportanceStore.add,
    usaf/moe_loader.py:604-611) for every expert with routed slots, without
    forming the dense gradient: three tensor-core SDDMM passes (exponent
    histogram, histogram inside the threshold bucket, emission) and device
    sorts.  Returns ``(vals, idx, experts)``: rows of ``k`` scores and flat
    indices ``e*R*C + r*C + c`` in ascending index order, one row per entry of
    ``experts`` (each row the set that a descending top-k with equal scores
    resolved to the lowest index keeps); or None when the fused path does not
    cover the shape or dtype (the caller then uses the dense |grad| path)."""
    if not _lib.LIB.usaf_importance_supported(R, C, dtc):
        return None
    dev = gout.device
    E = expert_cnt.numel()
    cnt_h = expert_cnt.cpu()
    experts = (cnt_h > 0).nonzero().reshape(-1)
    n_act = experts.numel()
    i32 = dict(dtype=torch.int32, device=dev)
    i64 = dict(dtype=torch.int64, device=dev)
    if n_act == 0:
        return (torch.empty(0, dtype=torch.float32, device=dev), torch.empty(0, **i64), experts)
    cand_row = torch.full((E,), -1, dtype=torch.int32)
    cand_row[experts] = torch.arange(n_act, dtype=torch.int32)
    cand_row = cand_row.to(dev)
    st = stream()
    hist = torch.zeros(E * 256, **i32)
    pval = torch.empty(E, **i32)
    need = torch.empty(E, **i64)
    thr = torch.empty(E, **i32)
    n_eq = torch.empty(E, **i64)
    args = (ptr(gout), ptr(gin), dtc)
    call("usaf_importance_hist", plan, R, C, *args, 1, None, ptr(hist), st)
    call("usaf_importance_pick", ptr(hist), E, k, ptr(expert_cnt), 1, ptr(pval), ptr(need), None, None, st)
    hist.zero_()
    call("usaf_importance_hist", plan, R, C, *args, 2, ptr(pval), ptr(hist), st)
    call("usaf_importance_pick", ptr(hist), E, k, None, 2, ptr(pval), ptr(need), ptr(thr), ptr(n_eq), st)
    eq_off = torch.cumsum(n_eq, 0) - n_eq
    n_ties = int(n_eq.sum())                       # host read: sizes the tie lists
    n = n_act * k
    vals = torch.empty(n, dtype=torch.float32, device=dev)
    idx = torch.empty(n, **i64)
    eq_val = torch.empty(max(n_ties, 1), dtype=torch.float32, device=dev)
    eq_idx = torch.empty(max(n_ties, 1), **i64)
    n_gt = torch.zeros(E, **i32)
    n_eqc = torch.zeros(E, **i32)
    call("usaf_importance_emit", plan, R, C, *args, ptr(thr), k, ptr(cand_row), ptr(n_gt), ptr(n_eqc),
         ptr(vals), ptr(idx), ptr(eq_off), ptr(eq_val), ptr(eq_idx), st)
    if n_ties:
        # ties at the threshold resolve to the lowest flat index: order the tie
        # lists by index and take each expert's first need[e]
        keys = torch.empty(n_ties, **i32)
        pos = torch.empty(n_ties, **i64)
        call("usaf_importance_keys", ptr(eq_val), ptr(eq_idx), None, n_ties, 1, 0, None, None, ptr(keys),
             ptr(pos), st)
        _, perm = sort_u32(keys, pos)
        ev, ei = torch.empty_like(eq_val), torch.empty_like(eq_idx)
        call("usaf_importance_keys", ptr(eq_val), ptr(eq_idx), ptr(perm), n_ties, 1, 2, ptr(ev), ptr(ei),
             None, None, st)
        call("usaf_importance_take_ties", E, k, ptr(cand_row), ptr(need), ptr(eq_off), ptr(ev), ptr(ei),
             ptr(vals), ptr(idx), st)
    # rows in ascending flat index order (the emission order is a race); the
    # flat index leads with the expert, so every row stays in place
    keys = torch.empty(n, **i32)
    pos = torch.empty(n, **i64)
    call("usaf_importance_keys", ptr(vals), ptr(idx), None, n, k, 0, None, None, ptr(keys), ptr(pos), st)
    _, perm = sort_u32(keys, pos)
    v1, i1 = torch.empty_like(vals), torch.empty_like(idx)
    call("usaf_importance_keys", ptr(vals), ptr(idx), ptr(perm), n, k, 2, ptr(v1), ptr(i1), None, None, st)
    return v1, i1, experts


def build_rowptr(rows: torch.Tensor, n_rows: int) -> torch.Tensor:
    rows = rows.to(torch.int64).contiguous()
    out = torch.empty(n_rows + 1, dtype=torch.int32, device=rows.device)
    call("usaf_build_rowptr", ptr(rows) if rows.numel() else None, rows.numel(), n_rows,
         ptr(out), stream())
    return out


def topk_desc(vals: torch.Tensor, k: int, idx_map: Optional[torch.Tensor] = None,
              idx_base: int = 0, want_vals: bool = True):
    """k largest of a 1-D fp32 tensor, descending; ties in ascending index order."""
    n = vals.numel()
    v = vals.contiguous().float()
    out_i = torch.empty(k, dtype=torch.int64, device=v.device)
    out_v = torch.empty(k, dtype=torch.float32, device=v.device) if want_vals else None
    scratch = torch.empty(int(_lib.LIB.usaf_topk_scratch_bytes(n, k)), dtype=torch.uint8,
                          device=v.device)
    call("usaf_topk_desc", ptr(v), n, k, ptr(idx_map), idx_base, ptr(out_v), ptr(out_i),
         ptr(scratch), stream())
    return out_v, out_i


def kth_largest(vals: torch.Tensor, k: int) -> torch.Tensor:
    n = vals.numel()
    v = vals.contiguous().float()
    out = torch.empty(1, dtype=torch.float32, device=v.device)
    scratch = torch.empty(int(_lib.LIB.usaf_topk_scratch_bytes(n, 1)), dtype=torch.uint8,
                          device=v.device)
    call("usaf_kth_largest", ptr(v), n, k, ptr(out), ptr(scratch), stream())
    return out


def _map(p) -> Optional[int]:
    """csr -> compact map of a projection for the gradient kernels (NULL = identity)."""
    return None if p.csr_identity else ptr(p.csr_to_compact)


def _check_act(name: str, t: torch.Tensor, shape, dtype: torch.dtype):
    """Shape / dtype / layout check of a tensor handed to the kernels: a wrong
    size would make them read or write past the buffer, so it raises here."""
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name}: expected shape {tuple(shape)}, got {tuple(t.shape)}")
    if t.dtype != dtype:
        raise TypeError(f"{name}: expected dtype {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")


def _bitmap(words: torch.Tensor, bits: torch.Tensor, n_words: int) -> torch.Tensor:
    """int32 words with bit ``bits[i]`` of word ``words[i]`` set (pairs distinct)."""
    m = torch.zeros(n_words, dtype=torch.int64, device=words.device)
    m.index_add_(0, words, torch.ones_like(bits) << bits)   # distinct bits: add == or
    return torch.where(m >= 2 ** 31, m - 2 ** 32, m).to(torch.int32)


class Projection:
    """One int4 expert projection resident in HBM, storage shape [E, R, C].

    ``q/s/z`` are the reference's packed codes, fp16 scales and zeros
    (usaf/quantization.py:21-85).  ``set_overlay(idx, master)`` installs the
    trained coordinates (flat indices into [E,R,C]) with their fp32 masters;
    the GEMMs then see ``dtype(fp16(master))`` at those coordinates, which is
    ``_get_resident`` + ``sync_resident`` of usaf/moe_loader.py:241-247, 442.
    """

    def __init__(self, q: torch.Tensor, s: torch.Tensor, z: torch.Tensor, shape,
                 group_size: int = 128, dtype: torch.dtype = torch.bfloat16):
        E, R, Cc = (int(x) for x in shape)
        if Cc % group_size != 0:
            raise ValueError("int4 groups must not straddle rows (C % group_size != 0)")
        if 2 * E * R * Cc >= 2 ** 32:
            raise ValueError("projection too large for 32-bit overlay keys")
        n_el = E * R * Cc
        # the usaf.quantization layout: 2 codes per byte, one fp16 scale and zero per group
        if q.numel() * 2 != n_el or q.dtype not in (torch.int8, torch.uint8):
            raise ValueError(f"q: expected {n_el // 2} int8 bytes for shape {tuple(shape)}, "
                             f"got {q.numel()} {q.dtype}")
        for nm, t in (("s", s), ("z", z)):
            if t.numel() != n_el // group_size or t.dtype != torch.float16:
                raise ValueError(f"{nm}: expected {n_el // group_size} fp16 values, "
                                 f"got {t.numel()} {t.dtype}")
        if not (q.device == s.device == z.device):
            raise ValueError("q, s and z must be on the same device")
        self.E, self.R, self.C, self.group_size = E, R, Cc, group_size
        self.shape = (E, R, Cc)
        self.q = q.reshape(-1).contiguous()
        self.s = s.reshape(-1).contiguous()
        self.z = z.reshape(-1).contiguous()
        self.dtype = dtype
        self.device = self.q.device
        self.n_ov = 0
        self.row_ptr = self.col = self.val = None
        self.colT_ptr = self.rowT = self.valT = None
        self.csr_to_compact = self.compact_to_csr = self.compact_to_csc = None
        self.csr_identity = False
        self.scratch = None
        self.ov_mask = self.ov_cbptr = None
        self.ov_emax = self.ov_emaxT = None
        self.qT = self.szT = self.qP = None
        if dtype == torch.bfloat16 and R % 8 == 0 and Cc % 8 == 0:
            # dequant-ordered copies for the tensor-core GEMMs (built once):
            # row-major for the forward, column-major for the backward
            self.qP = torch.empty_like(self.q)
            call("usaf_int4_repack", ptr(self.q), E * R * Cc, ptr(self.qP), stream())
            self.qT = torch.empty_like(self.q)
            self.szT = torch.empty(E * (Cc // group_size) * R, dtype=torch.int32, device=self.device)
            call("usaf_int4_transpose", ptr(self.q), ptr(self.s), ptr(self.z), E, R, Cc, group_size,
                 ptr(self.qT), ptr(self.szT), stream())
        self._struct = None

    def numel(self) -> int:
        return self.E * self.R * self.C

    def csr_order(self, idx: torch.Tensor) -> torch.Tensor:
        """Permutation that puts flat indices ``idx`` in the overlay's CSR order
        (row, 32-column half, column).  A caller that keeps its compact vectors
        in this order makes every compact <-> CSR map the identity, so the
        gradient scatter and the optimizer's overlay write-back stream."""
        idx = idx.reshape(-1).to(device=self.device, dtype=torch.int64)
        if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= self.numel()):
            # callers index the dequantized tensor with these next; refuse them here
            raise IndexError(f"active index out of range [0, {self.numel()})")
        E, R, Cc = self.E, self.R, self.C
        e = idx // (R * Cc)
        r = (idx // Cc) % R
        c = idx % Cc
        key = ((e * R + r) * 2 + ((c >> 5) & 1)) * Cc + c
        _, perm = sort_u32(key, torch.arange(idx.numel(), device=self.device, dtype=torch.int64))
        return perm.long()

    def set_overlay(self, idx: torch.Tensor, master: torch.Tensor):
        dev = self.device
        idx = idx.reshape(-1).to(device=dev, dtype=torch.int64)
        n = idx.numel()
        if master.numel() != n:
            raise ValueError(f"{master.numel()} master values for {n} overlay coordinates")
        if n and (int(idx.min()) < 0 or int(idx.max()) >= self.numel()):
            raise ValueError(f"overlay index out of range [0, {self.numel()})")
        E, R, Cc = self.E, self.R, self.C
        ar = torch.arange(n, device=dev, dtype=torch.int64)
        M32 = 0xFFFFFFFF
        e = idx // (R * Cc)
        r = (idx // Cc) % R
        c = idx % Cc
        # CSR: segments (row, half) with half = (col / 32) % 2, ascending col inside:
        # the tensor-core producers split every 64-wide k-block between two
        # threads per row, each walking its own sorted segment
        key = ((e * R + r) * 2 + ((c >> 5) & 1)) * Cc + c
        kcsr, pcsr = sort_u32(key, ar)
        if n > 1 and bool((kcsr[1:] == kcsr[:-1]).any()):
            raise ValueError("duplicate overlay coordinates")
        self.n_ov = n
        k64 = kcsr.to(torch.int64) & M32
        self.row_ptr = build_rowptr(k64 // Cc, E * R * 2)
        self.col = _i32(k64 % Cc)
        self.csr_to_compact = _i32(pcsr)
        # compact vectors kept in CSR order (the layers do): the kernels take the
        # identity map as NULL and stream instead of gathering
        self.csr_identity = bool(torch.equal(pcsr, ar))
        self.compact_to_csr = torch.empty(n, dtype=torch.int32, device=dev)
        self.compact_to_csr[pcsr] = torch.arange(n, device=dev, dtype=torch.int32)
        # CSC: segments (column, half) with half = (row / 32) % 2, ascending row
        keyT = ((e * Cc + c) * 2 + ((r >> 5) & 1)) * R + r
        kcsc, pcsc = sort_u32(keyT, ar)
        kc = kcsc.to(torch.int64) & M32
        self.colT_ptr = build_rowptr(kc // R, E * Cc * 2)
        self.rowT = _i32(kc % R)
        self.compact_to_csc = torch.empty(n, dtype=torch.int32, device=dev)
        self.compact_to_csc[pcsc] = torch.arange(n, device=dev, dtype=torch.int32)
        self._csc_to_compact = pcsc
        # bitmap of the selected coordinates, one 32-bit word per (row, 32 columns):
        # the tensor-core gradient epilogue reads a tile's selection from it
        self.ov_mask = self.ov_cbptr = None
        if Cc % 32 == 0:
            self.ov_mask = _bitmap((e * R + r) * (Cc // 32) + (c >> 5), c & 31, E * R * (Cc // 32))
            # first CSR position of every 256-column block of every segment: the
            # tensor-core epilogue starts a tile's writes there
            self.ov_cbptr = torch.empty(E * R * ((Cc + 255) // 256) * 2, dtype=torch.int32, device=dev)
            call("usaf_build_ov_cbptr", ptr(self.row_ptr), ptr(self.col), E, R, Cc, ptr(self.ov_cbptr),
                 stream())
        # per expert: the most trained storage row and column (work order of the GEMMs)
        self.ov_emax = (self.row_ptr[2::2] - self.row_ptr[:-1:2]).view(E, R).amax(1).to(torch.int32)
        self.ov_emaxT = (self.colT_ptr[2::2] - self.colT_ptr[:-1:2]).view(E, Cc).amax(1).to(torch.int32)
        self.val = torch.empty(n, dtype=torch.float32, device=dev)
        self.valT = torch.empty(n, dtype=torch.float32, device=dev)
        self.update_overlay_values(master)
        self.scratch = torch.empty(max(n, 1), dtype=torch.float32, device=dev)
        self._struct = None

    def update_overlay_values(self, master: torch.Tensor):
        ev = master.detach().to(self.device).half().to(self.dtype).float()
        self.val[self.compact_to_csr.long()] = ev
        self.valT[self.compact_to_csc.long()] = ev

    def struct(self) -> _lib.QWeight:
        if self._struct is None:
            st = _lib.QWeight()
            st.E, st.R, st.C, st.group_size = self.E, self.R, self.C, self.group_size
            st.q, st.s, st.z = ptr(self.q), ptr(self.s), ptr(self.z)
            st.n_ov = self.n_ov
            if self.n_ov:
                st.row_ptr, st.col, st.val = ptr(self.row_ptr), ptr(self.col), ptr(self.val)
                st.colT_ptr, st.rowT, st.valT = ptr(self.colT_ptr), ptr(self.rowT), ptr(self.valT)
            st.qT, st.szT, st.qP = ptr(self.qT), ptr(self.szT), ptr(self.qP)
            st.ov_mask = ptr(self.ov_mask) if (self.n_ov and self.ov_mask is not None) else None
            st.ov_cbptr = ptr(self.ov_cbptr) if (self.n_ov and self.ov_cbptr is not None) else None
            if self.n_ov:
                st.ov_emax, st.ov_emaxT = ptr(self.ov_emax), ptr(self.ov_emaxT)
            self._struct = st
        return self._struct

    def dequant(self, out_dtype=torch.float16) -> torch.Tensor:
        out = torch.empty(self.numel(), dtype=out_dtype, device=self.device)
        call("usaf_dequant_int4", ptr(self.q), ptr(self.s), ptr(self.z), self.numel(),
             self.group_size, _lib.dtype_code(out_dtype), ptr(out), stream())
        return out.view(self.shape)


@dataclass
class BlockDims:
    T: int
    H: int
    E: int
    I: int
    top_k: int
    norm_topk_prob: bool
    dtype: torch.dtype


def pair_capacity(T: int, E: int, top_k: int, pair_factor: float = 2) -> int:
    """Routed (token, expert) pairs a workspace holds: ``T * min(E,
    ceil(pair_factor * top_k))``.  Threshold ties route a token to more than
    top_k experts (usaf/qwen3moe_dml.py:79-80), so the default leaves room for
    twice top_k; a batch with more pairs is refused by the dispatch (error
    word, :meth:`MoEBlock.check`)."""
    if pair_factor < 1:
        raise ValueError("pair_factor must be >= 1 (every token routes to >= top_k experts)")
    return int(T) * min(int(E), int(math.ceil(pair_factor * top_k)))


class BackwardScratch:
    """Buffers a block uses only inside one call (its backward, and the
    router's GEMM scratch): the blocks of one model, whose forwards and
    backwards run one after another on one stream, can share one set.  Sized
    for ``P_cap`` pairs of T tokens; a block takes leading views."""

    def __init__(self, P_cap: int, T: int, H: int, E: int, I: int, dtype: torch.dtype, device):
        dev = torch.device(device)
        f32 = dict(dtype=torch.float32, device=dev)
        act = dict(dtype=dtype, device=dev)
        self.key = (int(P_cap), int(T), int(H), int(E), int(I), dtype, dev)
        self.dcur = torch.empty(P_cap, H, **act)
        self.dw_pair = torch.empty(P_cap, **f32)
        self.dgu = torch.empty(P_cap, 2 * I, **act)
        self.dx_seg = torch.empty(P_cap, H, **act)
        self.dlogits = torch.empty(T, E, **f32)
        self.dx_acc = torch.empty(T, H, **f32)
        self.dx = torch.empty(T, H, **act)
        self.dw_r = torch.empty(E, H, **act)
        self.router_ws = torch.empty(max(int(_lib.LIB.usaf_router_workspace_bytes(T, H, E)), 256),
                                     dtype=torch.uint8, device=dev)


class MoEBlock:
    """Workspace + kernel sequence of one MoE block step (single GPU).

    The pair buffers hold ``P_cap = pair_capacity(T, E, top_k, pair_factor)``
    routed (token, expert) pairs; threshold ties can route a token to more
    than top_k experts, and a batch that overflows the buffer is reported
    through the device error word (read by :meth:`check`).  ``scratch``
    (a :class:`BackwardScratch` of the same sizes) replaces the block's own
    backward-only buffers by a set shared with other blocks; the block's
    results (``dx``, ``dw_r``) then live in that set until the next block's
    backward, so callers copy them out (the autograd functions do).
    """

    def __init__(self, dims: BlockDims, device, pair_factor: float = 2,
                 scratch: Optional[BackwardScratch] = None):
        self.d = dims
        T, H, E, I = dims.T, dims.H, dims.E, dims.I
        self.device = torch.device(device)
        self.dt = dims.dtype
        self.dtc = _lib.dtype_code(dims.dtype)
        self.P_cap = pair_capacity(T, E, dims.top_k, pair_factor)
        dev, dt, Pc = self.device, self.dt, self.P_cap
        if scratch is None:
            scratch = BackwardScratch(Pc, T, H, E, I, dt, dev)
        elif scratch.key != (Pc, T, H, E, I, dt, dev):
            raise ValueError(f"shared scratch sized {scratch.key}, block needs "
                             f"{(Pc, T, H, E, I, dt, dev)}")
        self.scratch = scratch
        i32 = dict(dtype=torch.int32, device=dev)
        f32 = dict(dtype=torch.float32, device=dev)
        act = dict(dtype=dt, device=dev)
        nch = (T + 15) // 16     # dispatch chunks of 16 tokens
        self.tok_cnt = torch.zeros(max(T, 1), **i32)
        self.tok_off = torch.zeros(T + 1, **i32)
        self.expert_cnt = torch.zeros(E, **i32)
        self.expert_off = torch.zeros(E + 1, **i32)
        self.seg_tok = torch.zeros(Pc, **i32)
        self.seg_pair = torch.zeros(Pc, **i32)
        self.seg_w = torch.zeros(Pc, **f32)
        self.pair_exp = torch.zeros(Pc, **i32)
        self.pair_slot = torch.zeros(Pc, **i32)
        self.n_pairs = torch.zeros(1, **i32)
        self.chunk_cnt = torch.zeros(max(nch * E, 1), **i32)
        self.err = torch.zeros(1, **i32)
        self.sched = torch.zeros(16, **i32)      # GEMM work counters (kernels keep them zeroed)
        self.logits = torch.empty(T, E, **f32)
        self.probs = torch.empty(T, E, **f32)
        self.wsum = torch.empty(T, **f32)
        self.weights = torch.empty(T, E, **act)
        # kept from the forward for the backward
        self.x_perm = torch.empty(Pc, H, **act)
        self.gu = torch.empty(Pc, 2 * I, **act)
        self.h = torch.empty(Pc, I, **act)
        self.y_seg = torch.empty(Pc, H, **act)
        self.y = torch.empty(T, H, **act)
        # used inside one call only (possibly shared between blocks)
        self.dcur, self.dw_pair, self.dgu = scratch.dcur, scratch.dw_pair, scratch.dgu
        self.dx_seg, self.dlogits, self.dx_acc = scratch.dx_seg, scratch.dlogits, scratch.dx_acc
        self.dx, self.dw_r, self.router_ws = scratch.dx, scratch.dw_r, scratch.router_ws
        self.plan = _lib.RoutePlan()
        p = self.plan
        p.T, p.E, p.P_cap = T, E, Pc
        for name in ("tok_cnt", "tok_off", "expert_cnt", "expert_off", "seg_tok", "seg_pair",
                     "seg_w", "pair_exp", "pair_slot", "n_pairs", "chunk_cnt", "err", "sched"):
            setattr(p, name, ptr(getattr(self, name)))

    # ---------------------------------------------------------------- fwd ---
    def forward(self, x: torch.Tensor, w_r: torch.Tensor, gu: Projection, dn: Projection):
        d = self.d
        _check_act("x", x, (d.T, d.H), self.dt)
        _check_act("w_r", w_r, (d.E, d.H), self.dt)
        st = stream()
        call("usaf_router_fwd", ptr(x), ptr(w_r), self.dtc, d.T, d.H, d.E, d.top_k,
             int(d.norm_topk_prob), ptr(self.logits), ptr(self.probs), ptr(self.wsum),
             ptr(self.weights), ptr(self.router_ws), ptr(self.err), st)
        call("usaf_dispatch", self.plan, ptr(self.weights), ptr(x), self.dtc, d.H,
             ptr(self.x_perm), st)
        call("usaf_expert_gate_up_fwd", self.plan, gu.struct(), ptr(self.x_perm), self.dtc,
             ptr(self.gu), ptr(self.h), st)
        call("usaf_expert_down_fwd", self.plan, dn.struct(), ptr(self.h), self.dtc,
             ptr(self.y_seg), st)
        call("usaf_combine", self.plan, ptr(self.y_seg), self.dtc, d.H, ptr(self.y), st)
        return self.y

    # ---------------------------------------------------------------- bwd ---
    def backward(self, dy: torch.Tensor, x: torch.Tensor, w_r: torch.Tensor, gu: Projection,
                 dn: Projection):
        d = self.d
        _check_act("dy", dy, (d.T, d.H), self.dt)
        _check_act("x", x, (d.T, d.H), self.dt)
        _check_act("w_r", w_r, (d.E, d.H), self.dt)
        st = stream()
        call("usaf_combine_bwd", self.plan, ptr(dy), ptr(self.y_seg), self.dtc, d.H,
             ptr(self.dcur), ptr(self.dw_pair), st)
        call("usaf_router_bwd", self.plan, ptr(x), ptr(w_r), self.dtc, d.H,
             int(d.norm_topk_prob), ptr(self.probs), ptr(self.wsum), ptr(self.weights),
             ptr(self.dw_pair), ptr(self.dlogits), ptr(self.dw_r), ptr(self.dx_acc),
             ptr(self.router_ws), st)
        call("usaf_expert_down_bwd", self.plan, dn.struct(), ptr(self.dcur), ptr(self.gu),
             self.dtc, ptr(self.dgu), st)
        call("usaf_expert_gate_up_bwd", self.plan, gu.struct(), ptr(self.dgu), self.dtc,
             ptr(self.dx_seg), st)
        call("usaf_gather_dx", self.plan, ptr(self.dx_seg), ptr(self.dx_acc), self.dtc, d.H,
             ptr(self.dx), st)
        return self.dx, self.dw_r

    # ------------------------------------------ experts with given weights ---
    def experts_forward(self, x: torch.Tensor, weights: torch.Tensor, gu: Projection,
                        dn: Projection):
        """Expert part only: route by the dense [T, E] weights the caller
        gives (nonzero = routed), as ``dml_qwen3_experts_forward``
        (usaf/qwen3moe_dml.py:24-64) receives them."""
        d = self.d
        _check_act("x", x, (d.T, d.H), self.dt)
        _check_act("weights", weights, (d.T, d.E), self.dt)
        st = stream()
        self.weights.copy_(weights)
        call("usaf_dispatch", self.plan, ptr(self.weights), ptr(x), self.dtc, d.H,
             ptr(self.x_perm), st)
        call("usaf_expert_gate_up_fwd", self.plan, gu.struct(), ptr(self.x_perm), self.dtc,
             ptr(self.gu), ptr(self.h), st)
        call("usaf_expert_down_fwd", self.plan, dn.struct(), ptr(self.h), self.dtc,
             ptr(self.y_seg), st)
        call("usaf_combine", self.plan, ptr(self.y_seg), self.dtc, d.H, ptr(self.y), st)
        return self.y

    def experts_backward(self, dy: torch.Tensor, gu: Projection, dn: Projection):
        """Backward of :meth:`experts_forward`: (dX [T, H], dweights [T, E])."""
        d = self.d
        _check_act("dy", dy, (d.T, d.H), self.dt)
        st = stream()
        call("usaf_combine_bwd", self.plan, ptr(dy), ptr(self.y_seg), self.dtc, d.H,
             ptr(self.dcur), ptr(self.dw_pair), st)
        call("usaf_expert_down_bwd", self.plan, dn.struct(), ptr(self.dcur), ptr(self.gu),
             self.dtc, ptr(self.dgu), st)
        call("usaf_expert_gate_up_bwd", self.plan, gu.struct(), ptr(self.dgu), self.dtc,
             ptr(self.dx_seg), st)
        call("usaf_gather_dx", self.plan, ptr(self.dx_seg), None, self.dtc, d.H, ptr(self.dx), st)
        # d weights: pair p of token t and expert pair_exp[p] gets dw_pair[p]
        P = self.n_pairs_host()
        tok = torch.repeat_interleave(torch.arange(d.T, device=self.device),
                                      (self.tok_off[1:] - self.tok_off[:-1]).long(),
                                      output_size=P)
        dwts = torch.zeros(d.T, d.E, dtype=torch.float32, device=self.device)
        dwts[tok, self.pair_exp[:P].long()] = self.dw_pair[:P]
        return self.dx, dwts.to(self.dt)

    # ------------------------------------------------- expert weight grads ---
    def sparse_grads(self, gu: Projection, dn: Projection, compact_gu: torch.Tensor,
                     compact_dn: torch.Tensor, scale: float = 1.0):
        """compact[pos] += scale * dtype(dW[e,r,c]) at every overlay coordinate."""
        for nm, p, c in (("compact_gu", gu, compact_gu), ("compact_dn", dn, compact_dn)):
            if p.n_ov:
                _check_act(nm, c, (p.n_ov,), torch.float32)
        st = stream()
        if gu.n_ov:
            call("usaf_sparse_dw", self.plan, gu.struct(), ptr(self.dgu), ptr(self.x_perm),
                 self.dtc, _map(gu), scale, ptr(compact_gu), ptr(gu.scratch), st)
        if dn.n_ov:
            call("usaf_sparse_dw", self.plan, dn.struct(), ptr(self.dcur), ptr(self.h),
                 self.dtc, _map(dn), scale, ptr(compact_dn), ptr(dn.scratch), st)

    def hit_experts(self) -> torch.Tensor:
        """Experts with routed slots in the last forward."""
        return (self.expert_cnt > 0).nonzero().reshape(-1)

    def expert_candidates(self, which: str, k: int):
        """Per-expert top-``k`` |dW| candidates of one projection without the
        dense buffer (see :func:`expert_candidates`); None if not covered."""
        d = self.d
        if which == "gate_up_proj":
            R, Cc, gout, gin = 2 * d.I, d.H, self.dgu, self.x_perm
        else:
            R, Cc, gout, gin = d.H, d.I, self.dcur, self.h
        return expert_candidates(self.plan, self.expert_cnt, R, Cc, gout, gin, self.dtc, k)

    def dense_abs_grad(self, which: str) -> torch.Tensor:
        """|dW| of every expert of one projection as fp32 [E, R, C] (importance)."""
        d = self.d
        if which == "gate_up_proj":
            R, Cc, gout, gin = 2 * d.I, d.H, self.dgu, self.x_perm
        else:
            R, Cc, gout, gin = d.H, d.I, self.dcur, self.h
        out = torch.empty(d.E, R, Cc, dtype=torch.float32, device=self.device)
        call("usaf_expert_dense_dw", self.plan, R, Cc, ptr(gout), ptr(gin), self.dtc, ptr(out),
             stream())
        return out

    def check(self):
        """Raise if a kernel flagged an error (syncs the stream)."""
        e = int(self.err.item())
        if e:
            self.err.zero_()
            msgs = []
            if e & _lib.ERR_PAIR_OVERFLOW:
                msgs.append(f"routed pairs exceed the pair buffer ({self.P_cap})")
            if e & _lib.ERR_WAIT_TIMEOUT:
                msgs.append("a device-side wait timed out")
            if e & _lib.ERR_BAD_INDEX:
                msgs.append("an out-of-range index was skipped")
            raise _lib.UsafError("; ".join(msgs))

    def n_pairs_host(self) -> int:
        return int(self.n_pairs.item())


def sparse_adam_compact(master, m, v, grad, step, lr, betas, eps, weight_decay, proj=None,
                        grad_div=1.0, dtype=torch.bfloat16):
    """One fused SparseAdam step (usaf/sparse_optim.py:86-134, compact mode),
    writing the new overlay values of ``proj`` (sync_resident) in the same pass."""
    n = master.numel()
    for nm, t in (("master", master), ("m", m), ("v", v), ("grad", grad)):
        _check_act(nm, t, (n,), torch.float32)
    if proj is not None and proj.n_ov != n:
        raise ValueError(f"{n} masters for an overlay of {proj.n_ov} coordinates")
    call("usaf_sparse_adam", n, ptr(master), ptr(m), ptr(v), ptr(grad), float(grad_div),
         int(step), float(lr), float(betas[0]), float(betas[1]), float(eps),
         float(weight_decay), _lib.dtype_code(dtype),
         ptr(proj.val) if proj is not None else None,
         None if proj is None or proj.csr_identity else ptr(proj.compact_to_csr),
         ptr(proj.valT) if proj is not None else None,
         ptr(proj.compact_to_csc) if proj is not None else None, stream())


def sparse_adam_gather(param, grad, idx, m, v, step, lr, betas, eps, weight_decay,
                       grad_div=1.0):
    """SparseAdam gather/scatter mode (usaf/sparse_optim.py:110-134) on a
    dense parameter (the router)."""
    n = idx.numel()
    for nm, t in (("m", m), ("v", v)):
        _check_act(nm, t, (n,), torch.float32)
    if idx.dtype != torch.int64 or not idx.is_contiguous():
        raise TypeError("idx: contiguous int64 expected")
    if grad.numel() != param.numel() or grad.dtype != param.dtype or not grad.is_contiguous():
        raise ValueError("grad: a contiguous tensor of the parameter's size and dtype expected")
    call("usaf_sparse_adam_gather", n, ptr(idx), ptr(param), ptr(grad),
         _lib.dtype_code(param.dtype), float(grad_div), ptr(m), ptr(v), int(step), float(lr),
         float(betas[0]), float(betas[1]), float(eps), float(weight_decay), stream())
