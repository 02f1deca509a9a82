"""Multi-step parity of SparseMoELayer.train_step with the oracle.

Every step after the first reads the expert weights that the previous step's
fused SparseAdam wrote back into the overlays: the CSR copy read by the
forward GEMMs and the CSC copy read by the backward GEMMs
(``sync_resident`` then ``_get_resident`` on the next forward,
usaf/moe_loader.py:425-443 and :226-247).  The oracle rebuilds the effective
weights from its own masters at every step, so a write-back at a wrong
position or with a wrong rounding shows up from step 2 on.

Tolerances (relative Frobenius error): fp32 (C1) y, dX, dW_r, compact grads
<= 1e-5, masters <= 1e-6, router <= 1e-5; bf16 y, dX, dW_r, compact grads
<= 2e-2, and each step's master update (new master - old master) <= 2e-2:
Adam's m/sqrt(v) passes the bf16 gradients' rounding on to every update from
step 2 on, and the sign of g + wd * p flips where the two nearly cancel, so
the masters themselves carry the gradient tolerance, not 1e-6.  The learning rates are large enough that the
write-back moves the outputs by far more than these tolerances (checked on
the CPU in tests/test_oracle_trajectory.py).
"""
import numpy as np
import pytest
import torch

from oracle.flow import PREFIX, run_trajectory, step_dys
from oracle.inputs import C1, make_block_inputs

pytestmark = pytest.mark.gpu

GU, DN = f"{PREFIX}.gate_up_proj", f"{PREFIX}.down_proj"
MINI = dict(H=512, E=16, k=4, I=256, T=48, dtype=torch.bfloat16, seed=1, order="c2")
STEPS = 3


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def close(a, b, tol, what):
    r = rel(a, b)
    assert r <= tol, f"{what}: rel {r:.3e} > {tol:.1e}; max abs {(a.double().cpu()-b.double().cpu()).abs().max().item():.3e}"


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import usaf_b200  # noqa: F401
    return torch.device("cuda:0")


def random_active(inp, frac, seed):
    gen = torch.Generator().manual_seed(seed)
    E, H, I = inp["E"], inp["H"], inp["I"]
    out = {}
    for n, shape in ((GU, (E, 2 * I, H)), (DN, (E, H, I))):
        numel = int(np.prod(shape))
        out[n] = torch.randperm(numel, generator=gen)[: int(numel * frac)]
    return out


def device_trajectory(inp, dev, active, steps, lr, router_lr, router):
    from usaf_b200.engine import Projection
    from usaf_b200.layer import SparseMoELayer
    dtype = inp["dtype"]
    proj = {}
    for n in ("gate_up_proj", "down_proj"):
        e = inp[n]
        proj[n] = Projection(torch.from_numpy(e["q"]).to(dev), torch.from_numpy(e["s"]).to(dev),
                             torch.from_numpy(e["z"]).to(dev), e["shape"], 128, dtype)
    layer = SparseMoELayer(inp["w_r"].to(dev).contiguous().clone(), proj["gate_up_proj"],
                           proj["down_proj"], inp["k"], inp["T"], True, PREFIX)
    layer.init_selection({n: a.to(dev) for n, a in active.items()}, lr=lr, router_lr=router_lr,
                         router_optimizer=router)
    x = inp["x"].to(dev).contiguous()
    out = []
    for dy in step_dys(inp, steps):
        y, dx, dw_r = layer.train_step(x, dy.to(dev).contiguous())
        torch.cuda.synchronize()
        layer.block.check()
        rec = {"y": y.cpu().clone(), "dX": dx.cpu().clone(), "dW_r": dw_r.cpu().clone(),
               "weights": layer.block.weights.cpu().clone(),
               "compact": {n: layer.reorder_to(n, layer.store.compact[n], active[n]).cpu()
                           for n in active},
               "master_after": {n: layer.reorder_to(n, layer.masters[n], active[n]).cpu()
                                for n in active},
               "w_r_after": layer.w_r.cpu().clone()}
        if router == "sgd":
            rec["momentum"] = layer.router_sgd.state[layer.router_param]["momentum_buffer"].cpu().clone()
        out.append(rec)
    return out


CASES = {
    # C1 (fp32 SIMT kernels): golden-sized active set, router trained with SparseAdam
    "c1_adam": dict(cfg=C1, frac=0.005, lr=1e-3, router_lr=1e-3, router="adam"),
    # C1 with train.py's SGD-momentum router
    "c1_sgd": dict(cfg=C1, frac=0.005, lr=1e-3, router_lr=1e-2, router="sgd"),
    # bf16 (tcgen05 kernels): 5 % of the coordinates trained with a large step so the
    # written-back overlay moves y / dX far beyond the bf16 tolerance; the router is
    # frozen (lr 0) so that bf16 logit rounding cannot flip a route between the runs
    "mini_bf16": dict(cfg=MINI, frac=0.05, lr=1e-2, router_lr=0.0, router="sgd"),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_trajectory_vs_oracle(dev, case):
    c = CASES[case]
    cfg = c["cfg"]
    inp = make_block_inputs(**cfg)
    active = random_active(inp, c["frac"], seed=17)
    ref = run_trajectory(inp, active, STEPS, lr=c["lr"], router_lr=c["router_lr"],
                         router=c["router"])
    got = device_trajectory(inp, dev, active, STEPS, c["lr"], c["router_lr"], c["router"])
    fp32 = cfg["dtype"] == torch.float32
    tol = 1e-5 if fp32 else 2e-2
    # bf16: each step's master update (the SparseAdam step the overlay write-back
    # carries into the next step) is compared within the gradient tolerance
    from oracle.flow import masters_of
    start = masters_of(inp, active)
    prev_g = {n: start[n].clone() for n in (GU, DN)}
    prev_r = {n: start[n].clone() for n in (GU, DN)}
    for s, (g, r) in enumerate(zip(got, ref)):
        assert torch.equal(g["weights"] != 0, r["weights"] != 0), f"step {s}: routing differs"
        close(g["y"], r["y"], tol, f"step {s} y")
        close(g["dX"], r["dX"], tol, f"step {s} dX")
        close(g["dW_r"], r["dW_r"], tol, f"step {s} dW_r")
        for n in (GU, DN):
            close(g["compact"][n], r["compact"][n], tol, f"step {s} compact {n}")
            if fp32:
                close(g["master_after"][n], r["master_after"][n], 1e-6, f"step {s} master {n}")
                continue
            close(g["master_after"][n] - prev_g[n], r["master_after"][n] - prev_r[n], tol,
                  f"step {s} master update {n}")
            prev_g[n], prev_r[n] = g["master_after"][n], r["master_after"][n]
        if fp32:
            close(g["w_r_after"], r["w_r_after"], 1e-5, f"step {s} w_r_after")
            if c["router"] == "sgd":
                close(g["momentum"], r["momentum"], 1e-5, f"step {s} momentum")
        else:
            assert torch.equal(g["w_r_after"], inp["w_r"]), "router lr 0 must leave W_r unchanged"


def test_sgd_router_step_bf16(dev, golden_dir):
    """train.py's SGD-momentum router step (train.py:494-498, 667-672) on the
    bf16 mini case, two steps: the router's bf16 momentum buffer within the
    dW_r tolerance, and W_r off the oracle's by no more than what the two
    momentum buffers' difference moves it (lr * |buf_dev - buf_ref|) plus the
    bf16 rounding of the weight and of the update."""
    import os
    g = torch.load(os.path.join(golden_dir, "bf16_mini.pt"), weights_only=False)
    inp = make_block_inputs(**MINI)
    active = {GU: g[f"active.{GU}"], DN: g[f"active.{DN}"]}
    lr = 1e-3
    ref = run_trajectory(inp, active, 2, lr=1e-4, router_lr=lr, router="sgd")
    got = device_trajectory(inp, dev, active, 2, 1e-4, lr, "sgd")
    for s, (a, b) in enumerate(zip(got, ref)):
        assert torch.equal(a["weights"] != 0, b["weights"] != 0), f"step {s}: routing differs"
        close(a["momentum"].float(), b["momentum"].float(), 2e-2, f"step {s} momentum")
        w_a, w_b = a["w_r_after"].float(), b["w_r_after"].float()
        ba, bb = a["momentum"].float(), b["momentum"].float()
        # torch's CUDA SGD rounds w - lr * buf once, its CPU path may round the
        # update first: two bf16 roundings of |w| + |lr * buf| per step
        eps = torch.finfo(torch.bfloat16).eps
        upd = lr * torch.maximum(ba.abs(), bb.abs())
        bound = (lr * (ba - bb).abs() + 2 * eps * (torch.maximum(w_a.abs(), w_b.abs()) + upd)) * (s + 1)
        bad = (w_a - w_b).abs() > bound
        assert not bad.any(), f"step {s}: {int(bad.sum())} W_r entries off beyond the momentum difference"
        moved = (w_b != inp["w_r"].float()).float().mean().item()
        assert moved > 0.05, f"step {s}: the SGD step moved only {moved:.3f} of W_r"
