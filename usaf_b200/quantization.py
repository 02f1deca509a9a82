"""Packed int4 format of ``usaf.quantization`` on the device.

Same signatures and layout as the reference (usaf/quantization.py:21-132):
``quantize_4bit(tensor, group_size=128) -> (q int8 [G, ceil(gs/2)], s fp16 [G],
z fp16 [G], shape)`` and ``dequantize_4bit(q, s, z, shape, group_size=128) ->
fp16 tensor of ``shape```.  Both run the sm_100a kernels of
``csrc/quant.cu`` and are bit-exact with the reference; tensors must be on a
CUDA device.
"""
from __future__ import annotations

from typing import Any, Dict, Tuple

import torch

from . import _lib


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


def quantize_4bit(tensor: torch.Tensor, group_size: int = 128
                  ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Size]:
    if tensor.dim() == 0:
        raise ValueError("Scalar tensors cannot be quantized; skip them explicitly.")
    x = tensor.contiguous()
    if x.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        x = x.float()
    numel = x.numel()
    egs = min(group_size, numel)
    ng = (numel + egs - 1) // egs
    q = torch.empty((ng, (egs + 1) // 2), dtype=torch.int8, device=x.device)
    s = torch.empty(ng, dtype=torch.float16, device=x.device)
    z = torch.empty(ng, dtype=torch.float16, device=x.device)
    _lib.call("usaf_quant_int4", _lib.ptr(x), _lib.dtype_code(x.dtype), numel, group_size,
              _lib.ptr(q), _lib.ptr(s), _lib.ptr(z), _lib.stream())
    return q, s, z, tensor.shape


def dequantize_4bit(q_int4: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, shape,
                    group_size: int = 128, out_dtype: torch.dtype = torch.float16) -> torch.Tensor:
    numel = _numel(shape)
    # sizes of the quantize_4bit layout for this shape: the kernel reads exactly these
    egs = min(group_size, numel) if numel else group_size
    ng = (numel + egs - 1) // egs if numel else 0
    if q_int4.numel() != ng * ((egs + 1) // 2) or q_int4.dtype not in (torch.int8, torch.uint8):
        raise ValueError(f"q: expected {ng * ((egs + 1) // 2)} int8 bytes for shape {tuple(shape)} "
                         f"(group {group_size}), got {q_int4.numel()} {q_int4.dtype}")
    for nm, t in (("scale", scale), ("zero", zero)):
        if t.numel() != ng or t.dtype != torch.float16:
            raise ValueError(f"{nm}: expected {ng} fp16 values, got {t.numel()} {t.dtype}")
    out = torch.empty(numel, dtype=out_dtype, device=q_int4.device)
    # keep the contiguous copies alive until the kernel is enqueued
    q, s, z = q_int4.contiguous(), scale.contiguous(), zero.contiguous()
    _lib.call("usaf_dequant_int4", _lib.ptr(q), _lib.ptr(s), _lib.ptr(z), numel, group_size,
              _lib.dtype_code(out_dtype), _lib.ptr(out), _lib.stream())
    return out.view(tuple(shape))


def quantize_state_dict(state_dict: Dict[str, torch.Tensor], group_size: int = 128,
                        min_size: int = 256) -> Dict[str, Any]:
    """usaf/quantization.py:135-169 with the quantizer on the device."""
    out: Dict[str, Any] = {}
    for name, p in state_dict.items():
        if not isinstance(p, torch.Tensor):
            out[name] = p
        elif p.dim() == 0 or p.numel() < min_size:
            out[name] = p.detach().to(torch.float16)
        else:
            q, s, z, shape = quantize_4bit(p, group_size)
            out[name] = {"q": q, "s": s, "z": z, "shape": shape, "group_size": group_size}
    return out
