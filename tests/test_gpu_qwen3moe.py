"""The transformers Qwen3-MoE block patched by patch_qwen3moe_for_b200()
against the oracle's restatement of the reference block (oracle/moe.py
block_step = usaf/qwen3moe_dml.py:67-86 + autograd) on the same int4 weights
with an overlay of trained coordinates: output, dX, router gradient and the
compact expert gradients captured through the ``_grad_capture`` protocol.
Also the experts module called directly with dense routing weights, and the
importance capture (TopKImportanceStore) selecting the same coordinates.

Tolerance (bf16, as for the other block parity tests): relative Frobenius
error <= 2e-2 per tensor.
"""
import numpy as np
import pytest
import torch

from oracle import moe as omoe
from oracle import quant as oquant

pytestmark = pytest.mark.gpu

TOL = 2e-2
H, E, K, I, T = 512, 16, 4, 256, 96


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.fixture(scope="module")
def setup():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from usaf_b200 import qwen3moe
    from usaf_b200.engine import Projection
    mod = qwen3moe.patch_qwen3moe_for_b200()
    dev = torch.device("cuda:0")
    cfg = Qwen3MoeConfig(hidden_size=H, moe_intermediate_size=I, num_experts=E,
                         num_experts_per_tok=K, norm_topk_prob=True, hidden_act="silu")
    block = mod.Qwen3MoeSparseMoeBlock(cfg)
    g = torch.Generator().manual_seed(7)
    w_r = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    block.gate.weight.data = w_r.to(dev)
    block = block.to(dev)
    eff, projs, active = {}, {}, {}
    for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = (torch.randn(*shape, generator=g) * 0.02).numpy()
        q, s, z, _ = oquant.quantize_4bit(w, 128)
        numel = int(np.prod(shape))
        idx = torch.randperm(numel, generator=g)[: int(numel * 0.005)]
        master = torch.randn(idx.numel(), generator=g) * 0.02
        p = Projection(torch.from_numpy(q).to(dev), torch.from_numpy(s).to(dev),
                       torch.from_numpy(z).to(dev), shape, 128, torch.bfloat16)
        p.set_overlay(idx.to(dev), master.to(dev))
        projs[n], active[n] = p, idx
        deq = oquant.dequantize_4bit(q, s, z, shape, 128)
        eff[n] = omoe.effective_weight(deq, idx, master).reshape(shape).to(torch.bfloat16)
    qwen3moe.attach_int4_experts(block.experts, projs["gate_up_proj"], projs["down_proj"])
    x = torch.randn(2, T // 2, H, generator=g).to(torch.bfloat16)
    dy = torch.randn(2, T // 2, H, generator=g).to(torch.bfloat16)
    return dict(dev=dev, block=block, w_r=w_r, eff=eff, active=active, x=x, dy=dy, projs=projs)


def test_patched_block_vs_oracle(setup):
    from usaf_b200.moe_loader import SparseGradStore
    S = setup
    dev, block = S["dev"], S["block"]
    prefix = "model.layers.0.mlp.experts"
    names = {f"{prefix}.{n}": a for n, a in S["active"].items()}
    shapes = {f"{prefix}.gate_up_proj": (E, 2 * I, H), f"{prefix}.down_proj": (E, H, I)}
    store = SparseGradStore({n: a.to(dev) for n, a in names.items()}, shapes)
    block.experts._grad_capture = (store, prefix)
    block.gate.weight.grad = None
    x = S["x"].to(dev).requires_grad_(True)
    y = block(x)
    y.backward(S["dy"].to(dev))
    torch.cuda.synchronize()
    del block.experts._grad_capture

    ostore = omoe.SparseGradStore(names, shapes)
    ref = omoe.block_step(S["x"].reshape(-1, H), S["w_r"], S["eff"]["gate_up_proj"],
                          S["eff"]["down_proj"], S["dy"].reshape(-1, H), K, True,
                          capture=ostore.add, prefix=prefix, experts="dense")
    assert rel(y.detach().reshape(-1, H), ref["y"]) <= TOL
    assert rel(x.grad.reshape(-1, H), ref["dX"]) <= TOL
    assert rel(block.gate.weight.grad, ref["dW_r"]) <= TOL
    for n in names:
        assert rel(store.compact[n], ostore.compact[n]) <= TOL, n


def test_experts_direct_call_vs_oracle(setup):
    S = setup
    dev, block = S["dev"], S["block"]
    hs = S["x"].reshape(-1, H)
    _, _, _, weights = omoe.router_forward(hs.float().to(torch.bfloat16), S["w_r"], K, True)
    weights = weights.detach()
    h_dev = hs.to(dev).requires_grad_(True)
    w_dev = weights.to(dev).requires_grad_(True)
    y = block.experts(h_dev, w_dev)
    y.backward(S["dy"].reshape(-1, H).to(dev))
    hs_ref = hs.clone().requires_grad_(True)
    w_ref = weights.clone().requires_grad_(True)
    y_ref = omoe.experts_dense_masked(hs_ref, w_ref, S["eff"]["gate_up_proj"], S["eff"]["down_proj"])
    y_ref.backward(S["dy"].reshape(-1, H))
    assert rel(y.detach(), y_ref.detach()) <= TOL
    assert rel(h_dev.grad, hs_ref.grad) <= TOL
    # weights gradient only where routed (off-route entries are not pairs)
    m = weights != 0
    assert rel(w_dev.grad.cpu()[m], w_ref.grad[m]) <= TOL


def test_foreign_store_rejected(setup):
    S = setup
    block = S["block"]
    block.experts._grad_capture = ({}, "p")
    x = S["x"].to(S["dev"]).requires_grad_(True)
    with pytest.raises(TypeError):
        block(x).backward(S["dy"].to(S["dev"]))
    del block.experts._grad_capture
