"""Pins the CPU oracle against outputs of the reference implementation itself.

The fixtures in tests/golden were produced by tests/golden/make_golden.py,
which imports and runs the reference's own modules on the seeded inputs of
oracle.inputs.  These tests regenerate the inputs from the seed and check the
oracle against them: bit-exact for quantization, routing masks, dispatch
indices and selected coordinates; within the stated tolerance for floats.
"""
import hashlib
import os

import numpy as np
import pytest
import torch

from oracle import moe, quant
from oracle.flow import run_step, PREFIX
from oracle.inputs import make_block_inputs, C1

MINI = dict(H=512, E=16, k=4, I=256, T=48, dtype=torch.bfloat16, seed=1, order="c2")
GU, DN = f"{PREFIX}.gate_up_proj", f"{PREFIX}.down_proj"


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def load(golden_dir, name):
    return torch.load(os.path.join(golden_dir, name), weights_only=False)


@pytest.fixture(scope="module", params=["c1", "bf16_mini"])
def case(request, golden_dir):
    cfg = C1 if request.param == "c1" else MINI
    g = load(golden_dir, f"{request.param}.pt")
    inp = make_block_inputs(**cfg)
    return request.param, cfg, g, inp


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def test_quantization_matches_reference(case):
    _, _, g, inp = case
    for n in ("gate_up_proj", "down_proj"):
        e = inp[n]
        assert sha(e["q"], e["s"], e["z"]) == g[f"{n}.qsz_sha"]
        assert sha(e["fp16"]) == g[f"{n}.deq_sha"]


def test_flow_matches_reference_dense(case):
    """Dense-masked oracle: the reference's own operator sequence."""
    name, cfg, g, inp = case
    out = run_step(inp, experts="dense")
    assert torch.equal(out["weights"], g["weights"])
    for n in (GU, DN):
        assert torch.equal(out["active"][n], g[f"active.{n}"])
    assert torch.equal(out["y"], g["y"])
    assert torch.equal(out["dW_r"], g["dW_r"])
    assert rel(out["dX"], g["dX"]) < 1e-6
    for n in (GU, DN):
        assert torch.equal(out["compact"][n], g[f"compact.{n}"])
        assert torch.equal(out["master_after"][n], g[f"master_after.{n}"])
    assert torch.equal(out["w_r_after"], g["w_r_after"])


def test_flow_sparse_dispatch_within_tolerance(case):
    """The per-expert sparse loop (benchmarks/kaggle_t4_bench.py:253-282) is the
    oracle's fast mode; it must agree with the dense-masked reference."""
    name, cfg, g, inp = case
    out = run_step(inp, experts="sparse")
    tol = 1e-5 if cfg["dtype"] == torch.float32 else 2e-2
    assert torch.equal(out["weights"], g["weights"])
    assert rel(out["y"], g["y"]) < tol
    assert rel(out["dX"], g["dX"]) < tol
    assert rel(out["dW_r"], g["dW_r"]) < tol
    assert rel(out["y"], g["y_batched"]) < tol


def test_dispatch_indices_match_reference(case):
    _, _, g, inp = case
    d = moe.dispatch_indices(g["weights"])
    for key in ("tok_idx", "exp_idx", "counts", "order", "pos"):
        assert torch.equal(d[key], g[f"dispatch.{key}"]), key
    assert torch.equal(d["offs"], g["dispatch.offs"])


def test_router_ties_admit_more_than_k(golden_dir):
    t = load(golden_dir, "router_ties.pt")
    torch.manual_seed(t["seed"])
    w_r = (torch.randn(t["E"], t["H"]) * 0.02).to(torch.bfloat16)
    w_r[3] = w_r[1]
    w_r[5] = w_r[1]
    x = torch.randn(t["T"], t["H"]).to(torch.bfloat16)
    _, _, _, w = moe.router_forward(x, w_r, t["k"], True)
    assert torch.equal(w, t["weights"])
    assert int((w != 0).sum(1).max()) > t["k"]


def test_int4_known_answer():
    """Hand-computed pack/unpack of two groups of four (group_size=4)."""
    x = np.array([0.0, 1.0, 2.0, 3.0, -1.0, -1.0, 0.5, 2.0], np.float32)
    q, s, z, shape = quant.quantize_4bit(x, group_size=4)
    # group 0: min 0, scale 0.2 -> codes 0,5,10,15; group 1: min -1, scale 0.2 -> 0,0,7.5->8,15
    assert q.view(np.uint8).tolist() == [[0x50, 0xFA], [0x00, 0xF8]]
    assert np.allclose(s.astype(np.float32), [0.2, 0.2], atol=1e-4)
    assert z.tolist() == [0.0, -1.0]
    d = quant.dequantize_4bit(q, s, z, shape, 4)
    expect = (np.array([0, 5, 10, 15, 0, 0, 8, 15], np.float16).reshape(2, 4)
              * s[:, None] + z[:, None]).reshape(-1)
    assert np.array_equal(d, expect)


def test_adam_first_step_closed_form():
    """At t=1 with wd=0, |delta| = lr * |g| / (|g| + eps) (usaf/sparse_optim.py:123-127)."""
    g = torch.tensor([1e-3, -2.0, 5.0])
    m, v = torch.zeros(3), torch.zeros(3)
    d = moe.sparse_adam_update(torch.zeros(3), m, v, g, 1, lr=1e-4, weight_decay=0.0)
    assert torch.allclose(d.abs(), torch.full((3,), 1e-4), rtol=1e-4)
    assert torch.equal(torch.sign(d), -torch.sign(g))


def test_selector_known_answers():
    """Known answers of the reference's tests/test_selector.py:13-38."""
    s = {"a": torch.tensor([1.0, 2.0, 3.0, 4.0, 5.0]), "b": torch.tensor([0.1, 0.2, 0.3])}
    assert sum(int(m.sum()) for m in moe.topk_select(s, 3).values()) == 3
    assert int(moe.topk_select({"w": torch.tensor([1.0, 2.0, 3.0])}, 10)["w"].sum()) == 3
    m = moe.threshold_select({"w": torch.tensor([0.1, 0.5, 0.9, 1.0])}, 50.0)["w"]
    assert m.tolist() == [False, False, True, True]


def test_rigl_merge_known_answer():
    """train.py:559-596: kept sorted, grown = lowest new indices, grown values
    restart from the original dequant."""
    old = torch.tensor([9, 2, 5, 7])
    new = torch.tensor([5, 1, 8, 3, 9])
    masters = torch.tensor([90.0, 20.0, 50.0, 70.0])
    orig = torch.arange(10, dtype=torch.float16) * 0.5
    final, vals = moe.rigl_merge(old, new, masters, orig)
    assert final.tolist() == [5, 9, 1, 3]
    assert vals.tolist() == [50.0, 90.0, 0.5, 1.5]


@pytest.mark.parametrize("fname", ["t.gate_up_proj", "t.down_proj", "t.keep"])
def test_rigl_merge_matches_reference_fixture(golden_dir, fname):
    """The oracle's merge against the reference's own loop (train.py:552-596,
    extracted with ast and run by tests/golden/make_golden.py)."""
    g = load(golden_dir, "rigl.pt")
    inp = make_block_inputs(**C1)
    src = "gate_up_proj" if fname.endswith("gate_up_proj") else "down_proj"
    q, s, z, shape = quant.quantize_4bit(inp[src]["fp16"].astype(np.float32), 128)
    assert sha(q, s, z) == g[f"{fname}.qsz_sha"]
    orig = torch.from_numpy(quant.dequantize_4bit(q, s, z, shape, 128)).reshape(-1)
    new = g[f"{fname}.new"]
    final, vals = moe.rigl_merge(g[f"{fname}.old"], new, g[f"{fname}.masters"], orig)
    assert torch.equal(final.long(), g[f"{fname}.final"].long())
    assert torch.equal(vals.float(), g[f"{fname}.final_masters"])


def test_flow_batched_dispatch_matches_reference(case):
    """The oracle's restatement of the batched dispatch
    (benchmarks/kaggle_t4_bench.py:284-328, the CPU baseline's fast path):
    its output equals the reference function's own output on the same routing
    (the fixture ran the extracted reference function), and its training pass
    on the reference's active set agrees with the dense-masked reference
    within the float tolerance."""
    from oracle.flow import dense_weights, masters_of, shapes_of
    name, cfg, g, inp = case
    active = {n: g[f"active.{n}"] for n in (GU, DN)}
    masters = masters_of(inp, active)
    w_gu, w_dn = dense_weights(inp, {n: (active[n], masters[n]) for n in active})
    store = moe.SparseGradStore(active, shapes_of(inp))
    out = moe.block_step(inp["x"], inp["w_r"], w_gu, w_dn, inp["dy"], inp["k"], True,
                         capture=store.add, prefix=PREFIX, experts="batched")
    tol = 1e-5 if cfg["dtype"] == torch.float32 else 2e-2
    assert torch.equal(out["weights"], g["weights"])
    assert torch.equal(out["y"], g["y_batched"])
    assert rel(out["dX"], g["dX"]) < tol
    assert rel(out["dW_r"], g["dW_r"]) < tol
    for n in (GU, DN):
        assert rel(store.compact[n], g[f"compact.{n}"]) < tol
