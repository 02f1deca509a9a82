"""ctypes binding of the C ABI in include/usaf_b200.h.

The shared library is built in-tree (``python usaf_b200/build.py``).  There is
no fallback: importing an op without the library, or calling one on tensors
that are not on a CUDA device, raises.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libusaf_b200.so")

F32, BF16, F16 = 0, 1, 2
ERR_PAIR_OVERFLOW, ERR_WAIT_TIMEOUT, ERR_BAD_INDEX = 1, 2, 4
_STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported shape", 3: "CUDA launch failure"}

P = C.c_void_p
I32, I64, F32T, F64 = C.c_int32, C.c_int64, C.c_float, C.c_double


class RoutePlan(C.Structure):
    _fields_ = [("T", I32), ("E", I32), ("P_cap", I32),
                ("tok_cnt", P), ("tok_off", P), ("expert_cnt", P), ("expert_off", P),
                ("seg_tok", P), ("seg_pair", P), ("seg_w", P), ("pair_exp", P),
                ("pair_slot", P), ("n_pairs", P), ("chunk_cnt", P), ("err", P), ("sched", P)]


class QWeight(C.Structure):
    _fields_ = [("E", I32), ("R", I32), ("C", I32), ("group_size", I32),
                ("q", P), ("s", P), ("z", P), ("n_ov", I32),
                ("row_ptr", P), ("col", P), ("val", P),
                ("colT_ptr", P), ("rowT", P), ("valT", P), ("qT", P), ("szT", P), ("qP", P),
                ("ov_mask", P), ("ov_cbptr", P), ("ov_emax", P), ("ov_emaxT", P)]


# name -> (restype, argtypes)
_SIGS = {
    "usaf_dequant_int4": (I32, [P, P, P, I64, I32, I32, P, P]),
    "usaf_quant_int4": (I32, [P, I32, I64, I32, P, P, P, P]),
    "usaf_int4_transpose": (I32, [P, P, P, I32, I32, I32, I32, P, P, P]),
    "usaf_int4_repack": (I32, [P, I64, P, P]),
    "usaf_router_fwd": (I32, [P, P, I32, I32, I32, I32, I32, I32, P, P, P, P, P, P, P]),
    "usaf_router_workspace_bytes": (I64, [I32, I32, I32]),
    "usaf_router_select": (I32, [P, I32, I32, I32, I32, I32, P, P, P, P]),
    "usaf_router_bwd": (I32, [C.POINTER(RoutePlan), P, P, I32, I32, I32, P, P, P, P, P, P, P, P, P]),
    "usaf_dispatch": (I32, [C.POINTER(RoutePlan), P, P, I32, I32, P, P]),
    "usaf_combine": (I32, [C.POINTER(RoutePlan), P, I32, I32, P, P]),
    "usaf_combine_bwd": (I32, [C.POINTER(RoutePlan), P, P, I32, I32, P, P, P]),
    "usaf_gather_dx": (I32, [C.POINTER(RoutePlan), P, P, I32, I32, P, P]),
    "usaf_expert_gate_up_fwd": (I32, [C.POINTER(RoutePlan), C.POINTER(QWeight), P, I32, P, P, P]),
    "usaf_expert_down_fwd": (I32, [C.POINTER(RoutePlan), C.POINTER(QWeight), P, I32, P, P]),
    "usaf_expert_down_bwd": (I32, [C.POINTER(RoutePlan), C.POINTER(QWeight), P, P, I32, P, P]),
    "usaf_expert_gate_up_bwd": (I32, [C.POINTER(RoutePlan), C.POINTER(QWeight), P, I32, P, P]),
    "usaf_ep_permute": (I32, [P, I32, I32, I64, P, P, I64, I32, P, P]),
    "usaf_ep_owner_counts": (I32, [P, I32, I32, P, P, P, P]),
    "usaf_sparse_dw": (I32, [C.POINTER(RoutePlan), C.POINTER(QWeight), P, P, I32, P, F32T, P, P, P]),
    "usaf_sparse_dw_noalloc": (I32, [C.POINTER(RoutePlan), C.POINTER(QWeight), P, P, I32, P, F32T, P, P]),
    "usaf_expert_dense_dw": (I32, [C.POINTER(RoutePlan), I32, I32, P, P, I32, P, P]),
    "usaf_sparse_adam": (I32, [I64, P, P, P, P, F64, I32, F64, F64, F64, F64, F64, I32, P, P, P, P, P]),
    "usaf_sparse_adam_gather": (I32, [I64, P, P, P, I32, F64, P, P, I32, F64, F64, F64, F64, F64, P]),
    "usaf_topk_scratch_bytes": (I64, [I64, I64]),
    "usaf_topk_desc": (I32, [P, I64, I64, P, I64, P, P, P, P]),
    "usaf_kth_largest": (I32, [P, I64, I64, P, P, P]),
    "usaf_importance_chunk_slots": (I32, []),
    "usaf_importance_supported": (I32, [I32, I32, I32]),
    "usaf_importance_hist": (I32, [C.POINTER(RoutePlan), I32, I32, P, P, I32, I32, P, P, P]),
    "usaf_importance_pick": (I32, [P, I32, I64, P, I32, P, P, P, P, P]),
    "usaf_importance_emit": (I32, [C.POINTER(RoutePlan), I32, I32, P, P, I32, P, I64, P, P, P, P, P, P, P, P,
                                   P]),
    "usaf_importance_take_ties": (I32, [I32, I64, P, P, P, P, P, P, P, P]),
    "usaf_importance_keys": (I32, [P, P, P, I64, I64, I32, P, P, P, P, P]),
    "usaf_sort_scratch_bytes": (I64, [I64]),
    "usaf_sort_u32": (I32, [P, P, I64, P, P, I32, P, P]),
    "usaf_dot": (I32, [P, P, I32, I64, P, P]),
    "usaf_build_rowptr": (I32, [P, I64, I64, P, P]),
    "usaf_build_ov_cbptr": (I32, [P, P, I32, I32, I32, P, P]),
    "usaf_version": (C.c_char_p, []),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"usaf_b200 native library not found at {LIB_PATH}; build it with "
            "`python usaf_b200/build.py` (nvcc, sm_100a).  There is no CPU fallback.")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


LIB = _load()
EXPORTED = tuple(_SIGS)


class UsafError(RuntimeError):
    pass


def call(name: str, *args):
    rc = getattr(LIB, name)(*args)
    if rc != 0:
        raise UsafError(f"{name} failed: {_STATUS.get(rc, rc)} (status {rc})")


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return F32
    if dt == torch.bfloat16:
        return BF16
    if dt == torch.float16:
        return F16
    raise TypeError(f"unsupported dtype {dt}")


def ptr(t):
    """Device pointer of a CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not t.is_cuda:
        raise TypeError("usaf_b200 ops take CUDA tensors (no CPU fallback)")
    return t.data_ptr()


def stream():
    return torch.cuda.current_stream().cuda_stream
