"""Packed int4 quantize / dequantize restated in numpy (test oracle only).

Format (usaf/quantization.py:21-85): the tensor is flattened, split into
groups of ``min(group_size, numel)`` consecutive elements (zero padded at the
end), and each group stores
  * ``q``  int8 [groups, ceil(gs/2)]: two 4-bit codes per byte, the even
    element in the low nibble and the odd element in the high nibble;
  * ``s``  fp16 [groups]: scale = (max - min) / 15, clamped to >= 1e-12,
    computed in fp32 and then rounded to fp16;
  * ``z``  fp16 [groups]: zero = min, rounded to fp16.
Codes are ``clamp(round_half_even((x - min) / scale), 0, 15)`` with the fp32
(unrounded) scale and zero.  Dequantization (usaf/quantization.py:88-132)
computes ``fp16(fp16(q * s) + z)``: a half-precision multiply and a separate
half-precision add, each rounded.
"""
from __future__ import annotations

import numpy as np


def quantize_4bit(x, group_size: int = 128):
    """Restates ``quantize_4bit`` (usaf/quantization.py:21-85).

    ``x`` is any float array (converted to fp32 like ``tensor.flatten().float()``
    at :47).  Returns ``(q int8 [G, ceil(gs/2)], s fp16 [G], z fp16 [G], shape)``.
    """
    x = np.asarray(x)
    if x.ndim == 0:
        raise ValueError("Scalar tensors cannot be quantized; skip them explicitly.")
    shape = tuple(x.shape)
    flat = np.ascontiguousarray(x, dtype=np.float32).reshape(-1)
    numel = flat.size
    egs = min(group_size, numel)                                   # :50
    ng = (numel + egs - 1) // egs                                  # :51
    if ng * egs > numel:                                           # :54-55
        flat = np.concatenate([flat, np.zeros(ng * egs - numel, np.float32)])
    x2 = flat.reshape(ng, egs)
    mn = x2.min(axis=1, keepdims=True)                             # :59
    mx = x2.max(axis=1, keepdims=True)                             # :60
    scale = ((mx - mn) / np.float32(15.0)).astype(np.float32)      # :62
    scale = np.maximum(scale, np.float32(1e-12))                   # :63
    qf = np.rint((x2 - mn) / scale)                                # :66 (round half to even)
    qi = np.clip(qf, 0, 15).astype(np.uint8)                       # :67-68
    even = qi[:, 0::2]
    odd = np.zeros_like(even)
    if egs > 1:
        odd[:, : qi[:, 1::2].shape[1]] = qi[:, 1::2]               # :74-77
    packed = (even | (odd << 4)).astype(np.uint8).view(np.int8)    # :79-80
    return (np.ascontiguousarray(packed), scale[:, 0].astype(np.float16),
            mn[:, 0].astype(np.float16), shape)


def unpack_codes(q, numel: int, group_size: int = 128):
    """The 4-bit codes in element order (usaf/quantization.py:110-127)."""
    raw = np.asarray(q).view(np.uint8)
    ng, half = raw.shape
    inter = np.empty((ng, half * 2), np.uint8)
    inter[:, 0::2] = raw & 0x0F
    inter[:, 1::2] = (raw >> 4) & 0x0F
    egs = min(group_size, numel)
    return inter.reshape(-1)[: ng * egs].reshape(ng, egs)


def dequantize_4bit(q, s, z, shape, group_size: int = 128):
    """Restates ``dequantize_4bit`` (usaf/quantization.py:88-132); fp16 result."""
    numel = int(np.prod(shape)) if len(shape) else 1
    codes = unpack_codes(q, numel, group_size).astype(np.float16)
    prod = codes * np.asarray(s, np.float16)[:, None]              # fp16 multiply, :129
    out = prod + np.asarray(z, np.float16)[:, None]                # fp16 add, :129
    return out.reshape(-1)[:numel].reshape(shape)
