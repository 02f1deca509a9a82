"""Parity of the CUDA path (through the C ABI) with the CPU oracle and the
reference-generated golden fixtures.

Tolerances (relative Frobenius error, max-abs reported on failure):
  * bit-exact: int4 quantize/dequantize, routing weights given identical
    logits, dispatch indices, top-k selection given identical scores;
  * fp32 (C1): y, dX, dW_r, compact expert grads <= 1e-5; masters <= 1e-6;
  * bf16: y, dX, dW_r, compact grads <= 2e-2; masters <= 1e-6 (fp32 state).
"""
import os

import numpy as np
import pytest
import torch

from oracle import moe as omoe
from oracle import quant as oquant
from oracle.flow import PREFIX
from oracle.inputs import C1, make_block_inputs

pytestmark = pytest.mark.gpu

GU, DN = f"{PREFIX}.gate_up_proj", f"{PREFIX}.down_proj"
MINI = dict(H=512, E=16, k=4, I=256, T=48, dtype=torch.bfloat16, seed=1, order="c2")


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


def projections(inp, dev, dtype):
    from usaf_b200.engine import Projection
    out = {}
    for n in ("gate_up_proj", "down_proj"):
        e = inp[n]
        out[n] = Projection(torch.from_numpy(e["q"]).to(dev), torch.from_numpy(e["s"]).to(dev),
                            torch.from_numpy(e["z"]).to(dev), e["shape"], 128, dtype)
    return out


# ------------------------------------------------------------ int4 format --
@pytest.mark.parametrize("numel", [37, 128, 1000, 4096 * 3, 1 << 20])
def test_quant_dequant_bitexact(dev, numel):
    from usaf_b200.quantization import quantize_4bit, dequantize_4bit
    torch.manual_seed(numel)
    x = torch.randn(numel) * 0.02
    q, s, z, shape = oquant.quantize_4bit(x.numpy(), 128)
    qd, sd, zd, _ = quantize_4bit(x.to(dev), 128)
    assert np.array_equal(qd.cpu().numpy(), q)
    assert np.array_equal(sd.cpu().numpy().view(np.uint16), s.view(np.uint16))
    assert np.array_equal(zd.cpu().numpy().view(np.uint16), z.view(np.uint16))
    ref = oquant.dequantize_4bit(q, s, z, shape, 128)
    got = dequantize_4bit(qd, sd, zd, shape, 128).cpu().numpy()
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    got32 = dequantize_4bit(qd, sd, zd, shape, 128, out_dtype=torch.float32).cpu().numpy()
    assert np.array_equal(got32, ref.astype(np.float32))


def test_dequant_expert_tensor_bitexact(dev):
    inp = make_block_inputs(**MINI)
    p = projections(inp, dev, torch.bfloat16)
    for n in ("gate_up_proj", "down_proj"):
        got = p[n].dequant(torch.float16).cpu().numpy()
        assert np.array_equal(got.view(np.uint16), inp[n]["fp16"].view(np.uint16))


# ----------------------------------------------------------------- router --
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_router_select_bitexact_given_logits(dev, dtype):
    from usaf_b200 import _lib
    torch.manual_seed(3)
    T, E, H, k = 300, 128, 256, 8
    x = torch.randn(T, H).to(dtype)
    w = (torch.randn(E, H) * 0.02).to(dtype)
    logits, probs, mask, weights = omoe.router_forward(x, w, k, True)
    lg = logits.float().to(dev).contiguous()
    pr = torch.empty(T, E, device=dev)
    ws = torch.empty(T, device=dev)
    wt = torch.empty(T, E, dtype=dtype, device=dev)
    _lib.call("usaf_router_select", _lib.ptr(lg), _lib.dtype_code(dtype), T, E, k, 1,
              _lib.ptr(pr), _lib.ptr(ws), _lib.ptr(wt), _lib.stream())
    got_mask = (wt.cpu() != 0)
    assert torch.equal(got_mask, mask.bool() & (weights != 0))
    if dtype == torch.bfloat16:
        # equal bf16 logits -> equal probs: routing weights agree to 1 bf16 ulp
        diff = (wt.cpu().float() - weights.float()).abs()
        assert (diff <= weights.float().abs() * 2 ** -7).all()
    else:
        close(wt.cpu(), weights, 1e-6, "weights")
    close(pr.cpu(), probs, 1e-6, "probs")


def test_router_ties_fixture(dev, golden_dir):
    from usaf_b200 import _lib
    t = torch.load(os.path.join(golden_dir, "router_ties.pt"), weights_only=False)
    torch.manual_seed(t["seed"])
    w_r = (torch.randn(t["E"], t["H"]) * 0.02).to(torch.bfloat16)
    w_r[3] = w_r[1]
    w_r[5] = w_r[1]
    x = torch.randn(t["T"], t["H"]).to(torch.bfloat16)
    T, E, H = t["T"], t["E"], t["H"]
    lg = torch.empty(T, E, device=dev)
    pr = torch.empty(T, E, device=dev)
    ws = torch.empty(T, device=dev)
    wt = torch.empty(T, E, dtype=torch.bfloat16, device=dev)
    xd, wd = x.to(dev), w_r.to(dev)  # device copies must outlive the launch
    _lib.call("usaf_router_fwd", _lib.ptr(xd), _lib.ptr(wd), _lib.BF16, T, H, E,
              t["k"], 1, _lib.ptr(lg), _lib.ptr(pr), _lib.ptr(ws), _lib.ptr(wt), None, None, _lib.stream())
    assert torch.equal(wt.cpu() != 0, t["weights"] != 0)
    assert int((wt.cpu() != 0).sum(1).max()) > t["k"]


@pytest.mark.parametrize("E,H", [(8, 6144), (16, 512), (128, 2048)])
def test_router_logits_tensor_core_path(dev, E, H):
    """usaf_router_fwd with a workspace takes the tcgen05 GEMM (split-K partials
    summed in a fixed order, then one rounding to bf16); the logits agree with
    an fp32 product rounded to bf16 to one bf16 ulp, and the routing mask with
    the CUDA-core path (no workspace) wherever the two paths' logits agree."""
    from usaf_b200 import _lib
    torch.manual_seed(11)
    T, k = 300, 2 if E == 8 else 4
    x = torch.randn(T, H).to(torch.bfloat16)
    w_r = (torch.randn(E, H) * 0.02).to(torch.bfloat16)
    ref = (x.float() @ w_r.float().T).to(torch.bfloat16).float()
    xd, wd = x.to(dev), w_r.to(dev)
    ws = torch.empty(int(_lib.LIB.usaf_router_workspace_bytes(T, H, E)), dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    outs = []
    for wsp in (_lib.ptr(ws), None):
        lg = torch.empty(T, E, device=dev)
        pr = torch.empty(T, E, device=dev)
        wsum = torch.empty(T, device=dev)
        wt = torch.empty(T, E, dtype=torch.bfloat16, device=dev)
        _lib.call("usaf_router_fwd", _lib.ptr(xd), _lib.ptr(wd), _lib.BF16, T, H, E, k, 1,
                  _lib.ptr(lg), _lib.ptr(pr), _lib.ptr(wsum), _lib.ptr(wt), wsp,
                  _lib.ptr(err) if wsp is not None else None, _lib.stream())
        outs.append((lg.cpu(), wt.cpu()))
    assert int(err.item()) == 0
    (lg_tc, wt_tc), (lg_cc, wt_cc) = outs
    for lg in (lg_tc, lg_cc):
        assert ((lg - ref).abs() <= ref.abs() * 2 ** -7 + 1e-6).all()
    same = (lg_tc == lg_cc).all(1)
    assert same.float().mean() > 0.5
    assert torch.equal((wt_tc != 0)[same], (wt_cc != 0)[same])


# --------------------------------------------------------------- dispatch --
def test_dispatch_matches_reference_indices(dev, golden_dir):
    from usaf_b200.engine import BlockDims, MoEBlock
    from usaf_b200 import _lib
    g = torch.load(os.path.join(golden_dir, "bf16_mini.pt"), weights_only=False)
    w = g["weights"]
    T, E = w.shape
    blk = MoEBlock(BlockDims(T, 64, E, 128, 4, True, torch.bfloat16), dev)
    x = torch.randn(T, 64).to(torch.bfloat16).to(dev)
    wd = w.to(dev)
    _lib.call("usaf_dispatch", blk.plan, _lib.ptr(wd), _lib.ptr(x), _lib.BF16, 64,
              _lib.ptr(blk.x_perm), _lib.stream())
    P = blk.n_pairs_host()
    assert P == g["dispatch.tok_idx"].numel()
    assert torch.equal(blk.expert_cnt.cpu().long(), g["dispatch.counts"])
    assert torch.equal(blk.expert_off[:E].cpu().long(), g["dispatch.offs"])
    tok_sorted = g["dispatch.tok_idx"][g["dispatch.order"]]
    assert torch.equal(blk.seg_tok[:P].cpu().long(), tok_sorted)
    assert torch.equal(blk.pair_exp[:P].cpu().long(), g["dispatch.exp_idx"])
    assert torch.equal(blk.x_perm[:P].cpu(), x.cpu()[tok_sorted])


# -------------------------------------------------------------- selection --
def test_topk_bitexact_given_scores(dev):
    from usaf_b200.engine import topk_desc, kth_largest
    torch.manual_seed(0)
    v = torch.randn(1 << 18).abs()
    v[1000:1100] = v[5]  # ties
    k = 3000
    vals, idx = topk_desc(v.to(dev), k)
    order = sorted(range(v.numel()), key=lambda i: (-v[i].item(), i))[:k]
    assert idx.cpu().tolist() == order
    assert torch.equal(vals.cpu(), v[order])
    kth = kth_largest(v.to(dev), k).item()
    assert kth == float(np.partition(v.numpy(), v.numel() - k)[v.numel() - k])


# ------------------------------------------------------------ full flows --
def device_flow(inp, dev, active, lr=1e-4):
    """Our CUDA path on the oracle's inputs with a given active set."""
    from usaf_b200.layer import SparseMoELayer
    dtype = inp["dtype"]
    p = projections(inp, dev, dtype)
    w_r = inp["w_r"].to(dev).contiguous()
    layer = SparseMoELayer(w_r.clone(), p["gate_up_proj"], p["down_proj"], inp["k"], inp["T"],
                           True, PREFIX)
    x, dy = inp["x"].to(dev).contiguous(), inp["dy"].to(dev).contiguous()
    layer.init_selection({n: a.to(dev) for n, a in active.items()}, lr=lr)
    y, dx, dw_r = layer.train_step(x, dy)
    torch.cuda.synchronize()
    layer.block.check()
    return {"y": y.cpu().clone(), "dX": dx.cpu().clone(), "dW_r": dw_r.cpu().clone(),
            "weights": layer.block.weights.cpu().clone(),
            # the layer keeps compact vectors in CSR order: back to the caller's order
            "compact": {n: layer.reorder_to(n, layer.store.compact[n], active[n]).cpu() for n in active},
            "master_after": {n: layer.reorder_to(n, layer.masters[n], active[n]).cpu() for n in active},
            "w_r_after": layer.w_r.cpu().clone(), "layer": layer, "x": x, "dy": dy}


@pytest.mark.parametrize("case", ["c1", "bf16_mini"])
def test_flow_vs_golden(dev, golden_dir, case):
    cfg = C1 if case == "c1" else MINI
    g = torch.load(os.path.join(golden_dir, f"{case}.pt"), weights_only=False)
    inp = make_block_inputs(**cfg)
    active = {GU: g[f"active.{GU}"], DN: g[f"active.{DN}"]}
    out = device_flow(inp, dev, active)
    fp32 = cfg["dtype"] == torch.float32
    tol = 1e-5 if fp32 else 2e-2
    assert torch.equal(out["weights"] != 0, g["weights"] != 0)
    close(out["weights"].float(), g["weights"].float(), 1e-6 if fp32 else 1e-2, "weights")
    close(out["y"], g["y"], tol, "y")
    close(out["dX"], g["dX"], tol, "dX")
    close(out["dW_r"], g["dW_r"], tol, "dW_r")
    for n in (GU, DN):
        close(out["compact"][n], g[f"compact.{n}"], tol, f"compact {n}")
        close(out["master_after"][n], g[f"master_after.{n}"], 1e-6, f"master {n}")
    close(out["w_r_after"].float(), g["w_r_after"].float(), 1e-6 if fp32 else 1e-3, "w_r_after")


@pytest.mark.parametrize("case", ["c1", "bf16_mini"])
def test_importance_selection_vs_golden(dev, golden_dir, case):
    """Selection from the CUDA importance pass: the same number of coordinates,
    and every coordinate that differs from the reference's sits at a cut: its
    score is within the gradients' tolerance of the global k-th score or of
    its expert's candidate cut (the per-expert top-``2*frac`` of
    usaf/moe_loader.py:604-611).  Reference scores come from the fixture's
    candidate lists, device scores from the device store."""
    from usaf_b200.layer import SparseMoELayer
    cfg = C1 if case == "c1" else MINI
    g = torch.load(os.path.join(golden_dir, f"{case}.pt"), weights_only=False)
    inp = make_block_inputs(**cfg)
    p = projections(inp, dev, inp["dtype"])
    layer = SparseMoELayer(inp["w_r"].to(dev).contiguous(), p["gate_up_proj"], p["down_proj"],
                           inp["k"], inp["T"], True, PREFIX)
    store = layer.importance(inp["x"].to(dev).contiguous(), inp["dy"].to(dev).contiguous(), 0.005)
    sel = store.select(0.005)
    tol = 1e-5 if cfg["dtype"] == torch.float32 else 1e-2
    for n in (GU, DN):
        ref = g[f"active.{n}"]
        got = sel[n].cpu()
        assert got.numel() == ref.numel()
        numel_e = int(np.prod(p[n.rsplit(".", 1)[1]].shape[1:]))
        # score maps and cuts, reference side and device side
        r_vals, r_idx = g[f"cand.{n}.vals"].float(), g[f"cand.{n}.idx"].long()
        d_vals, d_idx = (t.cpu() for t in store.candidate_list(n))
        d_vals, d_idx = d_vals.float(), d_idx.long()
        sides = {"reference": (r_vals, r_idx, ref.long()), "device": (d_vals, d_idx, got.long())}
        cuts = {}
        for side, (vals, idx, chosen) in sides.items():
            score = dict(zip(idx.tolist(), vals.tolist()))
            kth = min(score[c] for c in chosen.tolist())
            per_e = {}
            for c, v in zip(idx.tolist(), vals.tolist()):
                e = c // numel_e
                per_e[e] = min(per_e.get(e, float("inf")), v)
            cuts[side] = (score, kth, per_e)
        only = {"reference": sorted(set(ref.tolist()) - set(got.tolist())),
                "device": sorted(set(got.tolist()) - set(ref.tolist()))}
        bad = []
        for side, coords in only.items():
            score, kth, per_e = cuts[side]
            for c in coords:
                v = score[c]
                near_kth = abs(v - kth) <= tol * kth
                near_cut = abs(v - per_e[c // numel_e]) <= tol * per_e[c // numel_e]
                if not (near_kth or near_cut):
                    bad.append((side, c, v, kth, per_e[c // numel_e]))
        n_diff = len(only["reference"])
        assert not bad, f"{n}: {len(bad)} of {n_diff} differing coordinates are not at a cut: {bad[:10]}"
        assert n_diff <= (0.001 if cfg["dtype"] == torch.float32 else 0.02) * ref.numel(), n_diff


def logit_flips(got_w, ref_w, ref_logits, k):
    """Tokens whose routing masks differ, with the reference's k-th and
    (k+1)-th largest bf16 logits and the bound a flip must respect: two
    logits that each carry at most one bf16 rounding of difference can only
    swap order (or tie) when they are within 2 ulp of each other."""
    flips = []
    tok = ((got_w != 0) != (ref_w != 0)).any(1).nonzero().reshape(-1).tolist()
    for t in tok:
        l = ref_logits[t].float().sort(descending=True).values
        a, b = l[k - 1].item(), l[k].item()
        mag = max(abs(a), abs(b), 2 ** -126)
        ulp = 2.0 ** (np.floor(np.log2(mag)) - 7)
        flips.append({"token": t, "kth": a, "next": b, "gap": a - b, "bound": 2 * ulp})
    return flips


def test_c2_shapes_vs_oracle(dev):
    """Qwen3-30B-A3B layer shapes (H 2048, E 128, k 8, I 768) at T=256, bf16,
    against the oracle's sparse-dispatch block on the same int4 weights."""
    from usaf_b200.quantization import quantize_4bit
    torch.manual_seed(1)
    H, E, k, I, T = 2048, 128, 8, 768, 256
    x = torch.randn(T, H).to(torch.bfloat16)
    w_r = (torch.randn(E, H) * 0.02).to(torch.bfloat16)
    inp = {"H": H, "E": E, "k": k, "I": I, "T": T, "dtype": torch.bfloat16, "x": x, "w_r": w_r,
           "dy": torch.randn(T, H).to(torch.bfloat16)}
    for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = (torch.randn(*shape, device=dev) * 0.02)
        q, s, z, _ = quantize_4bit(w, 128)
        inp[n] = {"q": q.cpu().numpy(), "s": s.cpu().numpy(), "z": z.cpu().numpy(), "shape": shape}
        inp[n]["fp16"] = oquant.dequantize_4bit(inp[n]["q"], inp[n]["s"], inp[n]["z"], shape, 128)
    gen = torch.Generator().manual_seed(5)
    active = {}
    for n, shape in ((GU, (E, 2 * I, H)), (DN, (E, H, I))):
        numel = int(np.prod(shape))
        active[n] = torch.randperm(numel, generator=gen)[: int(numel * 0.005)]
    out = device_flow(inp, dev, active)
    # oracle: same active set, same masters (original dequant), sparse dispatch
    from oracle.flow import dense_weights
    masters = {n: torch.from_numpy(inp[n.rsplit(".", 1)[1]]["fp16"].reshape(-1)[active[n].numpy()]).float()
               for n in active}
    w_gu, w_dn = dense_weights(inp, {n: (active[n], masters[n]) for n in active})
    shapes = {GU: (E, 2 * I, H), DN: (E, H, I)}
    store = omoe.SparseGradStore(active, shapes)
    ref = omoe.block_step(x, w_r, w_gu, w_dn, inp["dy"], k, True, capture=store.add,
                          prefix=PREFIX, experts="sparse")
    flips = logit_flips(out["weights"], ref["weights"], ref["logits"], k)
    print(f"routing flips ({len(flips)} of {T} tokens):", flips)
    wide = [f for f in flips if f["gap"] > f["bound"]]
    assert not wide, f"routing differs on tokens whose k-th/(k+1)-th logit gap exceeds 2 bf16 ulp: {wide}"
    keep = torch.ones(T, dtype=torch.bool)
    keep[[f["token"] for f in flips]] = False
    close(out["y"][keep], ref["y"][keep], 2e-2, "y")
    close(out["dX"][keep], ref["dX"][keep], 2e-2, "dX")
    close(out["dW_r"], ref["dW_r"], 2e-2, "dW_r")
    for n in (GU, DN):
        close(out["compact"][n], store.compact[n], 2e-2, f"compact {n}")


def test_c2_full_step_vs_oracle(dev):
    """The benched configuration itself: one C2 layer (T 4096, H 2048, E 128,
    k 8, I 768, bf16), overlay chosen by the device importance pass (rows with
    hundreds of trained coordinates), one train_step against the oracle's
    sparse-dispatch block on the same int4 weights and active set.  Routing
    flips are listed and must sit within 2 bf16 ulp of a logit tie; y and dX
    are compared on the other tokens."""
    from usaf_b200.engine import Projection
    from usaf_b200.layer import SparseMoELayer
    from usaf_b200.quantization import quantize_4bit
    from oracle.flow import dense_weights
    H, E, k, I, T = 2048, 128, 8, 768, 4096
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    w_r = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    dy = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    inp = {"H": H, "E": E, "k": k, "I": I, "T": T, "dtype": torch.bfloat16,
           "x": x.cpu(), "w_r": w_r.cpu(), "dy": dy.cpu()}
    proj = {}
    for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = torch.randn(*shape, device=dev, generator=g) * 0.02
        q, s, z, _ = quantize_4bit(w, 128)
        del w
        proj[n] = Projection(q, s, z, shape, 128, torch.bfloat16)
        # the device dequant is bit-exact with the oracle's (test_dequant_expert_tensor_bitexact)
        inp[n] = {"shape": shape, "fp16": proj[n].dequant(torch.float16).cpu().numpy()}
    layer = SparseMoELayer(w_r.clone(), proj["gate_up_proj"], proj["down_proj"], k, T, True, PREFIX)
    active = {n: a.cpu() for n, a in layer.importance(x, dy, 0.005).select(0.005).items()}
    layer.init_selection({n: a.to(dev) for n, a in active.items()}, lr=1e-4)
    y, dx, dw_r = layer.train_step(x, dy)
    torch.cuda.synchronize()
    layer.block.check()
    out = {"y": y.cpu(), "dX": dx.cpu(), "dW_r": dw_r.cpu(), "weights": layer.block.weights.cpu(),
           "compact": {n: layer.reorder_to(n, layer.store.compact[n], active[n].to(dev)).cpu()
                       for n in active}}
    masters = {n: torch.from_numpy(inp[n.rsplit(".", 1)[1]]["fp16"].reshape(-1)[active[n].numpy()]).float()
               for n in active}
    w_gu, w_dn = dense_weights(inp, {n: (active[n], masters[n]) for n in active})
    shapes = {GU: (E, 2 * I, H), DN: (E, H, I)}
    store = omoe.SparseGradStore(active, shapes)
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    ref = omoe.block_step(inp["x"], inp["w_r"], w_gu, w_dn, inp["dy"], k, True, capture=store.add,
                          prefix=PREFIX, experts="sparse")
    flips = logit_flips(out["weights"], ref["weights"], ref["logits"], k)
    print(f"C2 routing flips ({len(flips)} of {T} tokens):", flips)
    wide = [f for f in flips if f["gap"] > f["bound"]]
    assert not wide, f"routing differs on tokens whose k-th/(k+1)-th logit gap exceeds 2 bf16 ulp: {wide}"
    keep = torch.ones(T, dtype=torch.bool)
    keep[[f["token"] for f in flips]] = False
    close(out["y"][keep], ref["y"][keep], 2e-2, "y")
    close(out["dX"][keep], ref["dX"][keep], 2e-2, "dX")
    close(out["dW_r"], ref["dW_r"], 2e-2, "dW_r")
    for n in (GU, DN):
        close(out["compact"][n], store.compact[n], 2e-2, f"compact {n}")
