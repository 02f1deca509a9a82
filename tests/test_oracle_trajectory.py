"""The oracle's multi-step trajectory (oracle.flow.run_trajectory), on the CPU.

* Its first step is the reference's own step: with the golden active sets,
  SparseAdam router and the dense-masked experts it reproduces the fixtures
  that tests/golden/make_golden.py made by running the reference, bit for bit.
* The device trajectory test (tests/test_gpu_trajectory.py) can see a broken
  overlay write-back: a trajectory whose overlays stay at the initial masters
  (a planted fault, here in the oracle) differs from the real one at step 2 by
  far more than that test's tolerances.
"""
import os

import numpy as np
import pytest
import torch

from oracle.flow import PREFIX, run_trajectory
from oracle.inputs import C1, make_block_inputs

GU, DN = f"{PREFIX}.gate_up_proj", f"{PREFIX}.down_proj"
MINI = dict(H=512, E=16, k=4, I=256, T=48, dtype=torch.bfloat16, seed=1, order="c2")


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("case", ["c1", "bf16_mini"])
def test_first_step_is_the_reference_step(golden_dir, case):
    cfg = C1 if case == "c1" else MINI
    g = torch.load(os.path.join(golden_dir, f"{case}.pt"), weights_only=False)
    inp = make_block_inputs(**cfg)
    active = {GU: g[f"active.{GU}"], DN: g[f"active.{DN}"]}
    r = run_trajectory(inp, active, 1, lr=1e-4, router="adam", experts="dense")[0]
    assert torch.equal(r["y"], g["y"])
    assert torch.equal(r["dW_r"], g["dW_r"])
    for n in (GU, DN):
        assert torch.equal(r["compact"][n], g[f"compact.{n}"])
        assert torch.equal(r["master_after"][n], g[f"master_after.{n}"])
    assert torch.equal(r["w_r_after"], g["w_r_after"])


def _active(inp, frac, seed):
    gen = torch.Generator().manual_seed(seed)
    E, H, I = inp["E"], inp["H"], inp["I"]
    out = {}
    for n, shape in ((GU, (E, 2 * I, H)), (DN, (E, H, I))):
        numel = int(np.prod(shape))
        out[n] = torch.randperm(numel, generator=gen)[: int(numel * frac)]
    return out


@pytest.mark.parametrize("cfg,frac,lr,router_lr,router,tol", [
    (C1, 0.005, 1e-3, 1e-3, "adam", 1e-5),
    (C1, 0.005, 1e-3, 1e-2, "sgd", 1e-5),
    (MINI, 0.05, 1e-2, 0.0, "sgd", 2e-2),
])
def test_lost_write_back_is_visible(cfg, frac, lr, router_lr, router, tol):
    inp = make_block_inputs(**cfg)
    active = _active(inp, frac, seed=17)
    good = run_trajectory(inp, active, 2, lr=lr, router_lr=router_lr, router=router)
    bad = run_trajectory(inp, active, 2, lr=lr, router_lr=router_lr, router=router,
                         write_back=False)
    assert torch.equal(good[0]["y"], bad[0]["y"])          # step 1 reads the initial masters
    for key in ("y", "dX"):
        assert rel(bad[1][key], good[1][key]) > 10 * tol, key
