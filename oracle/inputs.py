"""Seeded synthetic inputs of the benchmark configurations (test oracle only).

The reference publishes no dataset for this path; every configuration is a
seeded synthetic draw.  Generation happens once on the CPU and the same
tensors feed both the oracle and the CUDA path.

* C1: ``torch.manual_seed(0)``; W_r [E,H], W_gu [E,2I,H], W_dn [E,H,I] ~ N(0, 0.02)
  drawn in that order, then X [T,H] ~ N(0,1) and the upstream gradient
  dY [T,H] ~ N(0,1); fp32.
* C2-shaped (bf16): ``torch.manual_seed(seed)``; X, W_r, W_gu, W_dn, dY in that
  order, drawn in fp32 and rounded to bf16 (weights are quantized from fp32).
* Zipf routing (C4): the constant feature ``X[:,0] = 1`` and ``log p_e`` with
  ``p_e ~ rank_e^-s`` (normalised) added to ``W_r[:,0]``, so the router's logits
  carry a per-expert bias through the reference's bias-free router.
"""
from __future__ import annotations

import numpy as np
import torch

from .quant import quantize_4bit, dequantize_4bit


def zipf_log_bias(E: int, s: float) -> torch.Tensor:
    p = np.arange(1, E + 1, dtype=np.float64) ** (-s)
    p /= p.sum()
    return torch.from_numpy(np.log(p)).float()


def make_block_inputs(H, E, k, I, T, dtype=torch.bfloat16, seed=1, order="c2",
                      zipf_s=None, std=0.02, group_size=128, with_dense=True):
    torch.manual_seed(seed)
    if order == "c1":
        w_r = torch.randn(E, H) * std
        w_gu = torch.randn(E, 2 * I, H) * std
        w_dn = torch.randn(E, H, I) * std
        x = torch.randn(T, H)
        dy = torch.randn(T, H)
    else:
        x = torch.randn(T, H)
        w_r = torch.randn(E, H) * std
        w_gu = torch.randn(E, 2 * I, H) * std
        w_dn = torch.randn(E, H, I) * std
        dy = torch.randn(T, H)
    if zipf_s is not None:
        x[:, 0] = 1.0
        w_r[:, 0] += zipf_log_bias(E, zipf_s)
    out = {"H": H, "E": E, "k": k, "I": I, "T": T, "dtype": dtype,
           "x": x.to(dtype), "w_r": w_r.to(dtype), "dy": dy.to(dtype)}
    for name, w in (("gate_up_proj", w_gu), ("down_proj", w_dn)):
        q, s, z, shape = quantize_4bit(w.numpy(), group_size)
        out[name] = {"q": q, "s": s, "z": z, "shape": shape, "group_size": group_size}
        if with_dense:
            out[name]["fp16"] = dequantize_4bit(q, s, z, shape, group_size)
    return out


C1 = dict(H=256, E=8, k=2, I=512, T=64, dtype=torch.float32, seed=0, order="c1")
C2 = dict(H=2048, E=128, k=8, I=768, T=4096, dtype=torch.bfloat16, seed=1, order="c2")
