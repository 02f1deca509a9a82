"""Grouped expert GEMM kernels against a plain torch fp32 reference of the
same op (dequantized int4 weights with the overlay applied, computed per
expert segment in fp32, rounded to bf16).

Tolerance: the kernels accumulate in fp32 in a different order, so results
agree to bf16 rounding: max |diff| <= 2 bf16 ulps of the reference value
(4 for the SwiGLU-backward gate gradient, which passes through two rounded
intermediates), plus 1e-3 absolute slack for values near zero, and relative
Frobenius error <= 4e-3.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import usaf_b200  # noqa: F401
    return torch.device("cuda:0")


def make_case(dev, T, H, E, k, I, zipf=None, seed=0, ov_frac=0.005, skew=False):
    from usaf_b200.engine import BlockDims, MoEBlock, Projection
    from usaf_b200.quantization import quantize_4bit
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    w_r = (torch.randn(E, H, device=dev, generator=g) * 0.02)
    if zipf is not None:
        x[:, 0] = 1.0
        p = torch.arange(1, E + 1, device=dev, dtype=torch.float64) ** (-zipf)
        w_r[:, 0] += torch.log(p / p.sum()).float()
    w_r = w_r.to(torch.bfloat16)
    projs = {}
    for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = torch.randn(*shape, device=dev, generator=g) * 0.02
        q, s, z, _ = quantize_4bit(w, 128)
        p_ = Projection(q, s, z, shape, 128, torch.bfloat16)
        numel = p_.numel()
        n_ov = max(1, int(numel * ov_frac))
        if numel > 1 << 28:   # large tensors: random draws + unique (a full permutation is slow)
            idx = torch.unique(torch.randint(0, numel, (n_ov,), device=dev, generator=g))
            idx = idx[torch.randperm(idx.numel(), device=dev, generator=g)]
        else:
            idx = torch.randperm(numel, device=dev, generator=g)[:n_ov]
        if skew:
            # whole storage rows and columns selected: 32 coordinates in one
            # 32-wide half block, for the forward and for the transposed backward
            Rr, Cc = shape[1], shape[2]
            rows = torch.randint(0, E * Rr, (3,), device=dev, generator=g)
            cols = torch.randint(0, Cc, (3,), device=dev, generator=g)
            ee = torch.randint(0, E, (3,), device=dev, generator=g)
            heavy_r = (rows[:, None] * Cc + torch.arange(Cc, device=dev)[None, :]).reshape(-1)
            heavy_c = ((ee[:, None] * Rr + torch.arange(Rr, device=dev)[None, :]) * Cc + cols[:, None]).reshape(-1)
            idx = torch.unique(torch.cat([idx, heavy_r, heavy_c]))
            idx = idx[torch.randperm(idx.numel(), device=dev, generator=g)]
        master = (torch.randn(idx.numel(), device=dev, generator=g) * 0.05)
        p_.set_overlay(idx, master)
        projs[n] = p_
    blk = MoEBlock(BlockDims(T, H, E, I, k, True, torch.bfloat16), dev)
    return blk, x, w_r, projs


def eff_weight(p):
    w = p.dequant(torch.float16).reshape(-1).clone()
    idx = torch.empty(p.n_ov, dtype=torch.long, device=w.device)
    # reconstruct the overlay flat indices from the CSR
    rows = torch.repeat_interleave(torch.arange(p.E * p.R * 2, device=w.device) // 2,
                                   (p.row_ptr[1:] - p.row_ptr[:-1]).long())
    idx = rows * p.C + p.col.long()
    w[idx] = p.val.to(torch.float16)
    return w.view(p.shape).to(torch.bfloat16).float()


def check(got, ref, what, ulps=2):
    got, ref = got.float(), ref.float()
    ulp = ref.abs() * 2 ** -7 * ulps + 1e-3
    bad = (got - ref).abs() > ulp
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    assert not bad.any(), f"{what}: {int(bad.sum())} elems beyond {ulps} ulp; rel {rel:.2e}"
    assert rel <= 4e-3, f"{what}: rel {rel:.2e}"


CASES = [
    dict(T=256, H=512, E=16, k=4, I=256),
    dict(T=1, H=512, E=16, k=4, I=256),
    dict(T=17, H=512, E=16, k=4, I=256),
    dict(T=2048, H=512, E=16, k=4, I=256, zipf=1.2),   # skewed: experts > 384 tokens
    dict(T=512, H=2048, E=128, k=8, I=768),            # Qwen3-30B-A3B layer shapes
    dict(T=256, H=512, E=16, k=4, I=256, skew=True),   # fully selected rows and columns
    # C4 sweep points at the Qwen3-30B-A3B shapes (T=1, 16, 256 are covered above at
    # small H; 4096 with Zipf(1.2) routing, 16384 uniform)
    dict(T=4096, H=2048, E=128, k=8, I=768, zipf=1.2),
    dict(T=16384, H=2048, E=128, k=8, I=768),
    # C5: Mixtral-8x22B-shaped experts (E=8, top-2, H=6144, I=16384)
    dict(T=256, H=6144, E=8, k=2, I=16384),
    # decode-sized plans at the layer shapes: one token, 16 spread over the experts,
    # 32 on a few experts, fully selected rows with few tokens, C5 experts
    dict(T=1, H=2048, E=128, k=8, I=768),
    dict(T=16, H=2048, E=128, k=8, I=768),
    dict(T=32, H=2048, E=128, k=8, I=768, zipf=1.2),
    dict(T=8, H=512, E=16, k=4, I=256, skew=True),
    dict(T=4, H=6144, E=8, k=2, I=16384),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "T{T}_H{H}_E{E}_I{I}".format(**c) + ("_zipf" if "zipf" in c else "") + ("_skew" if c.get("skew") else ""))
def test_grouped_gemms_vs_torch(dev, case):
    from usaf_b200 import _lib
    blk, x, w_r, p = make_case(dev, **case)
    st = _lib.stream()
    _lib.call("usaf_router_fwd", _lib.ptr(x), _lib.ptr(w_r), _lib.BF16, case["T"], case["H"],
              case["E"], case["k"], 1, _lib.ptr(blk.logits), _lib.ptr(blk.probs),
              _lib.ptr(blk.wsum), _lib.ptr(blk.weights), _lib.ptr(blk.router_ws), _lib.ptr(blk.err), st)
    _lib.call("usaf_dispatch", blk.plan, _lib.ptr(blk.weights), _lib.ptr(x), _lib.BF16, case["H"],
              _lib.ptr(blk.x_perm), st)
    _lib.call("usaf_expert_gate_up_fwd", blk.plan, p["gate_up_proj"].struct(), _lib.ptr(blk.x_perm),
              _lib.BF16, _lib.ptr(blk.gu), _lib.ptr(blk.h), st)
    _lib.call("usaf_expert_down_fwd", blk.plan, p["down_proj"].struct(), _lib.ptr(blk.h), _lib.BF16,
              _lib.ptr(blk.y_seg), st)
    torch.cuda.synchronize()
    blk.check()
    P = blk.n_pairs_host()
    off = blk.expert_off.cpu().tolist()
    cnt = blk.expert_cnt.cpu().tolist()
    wgu, wdn = eff_weight(p["gate_up_proj"]), eff_weight(p["down_proj"])
    I = case["I"]
    gu_ref = torch.empty(P, 2 * I, device=dev)
    y_ref = torch.empty(P, case["H"], device=dev)
    for e in range(case["E"]):
        if cnt[e] == 0:
            continue
        sl = slice(off[e], off[e] + cnt[e])
        gu_ref[sl] = (blk.x_perm[sl].float() @ wgu[e].T).to(torch.bfloat16).float()
        # down input = the kernel's own h (checked separately below)
        y_ref[sl] = (blk.h[sl].float() @ wdn[e].T).to(torch.bfloat16).float()
    check(blk.gu[:P], gu_ref, "gate_up")
    g, u = blk.gu[:P, :I].float(), blk.gu[:P, I:].float()
    s = (g / (1 + torch.exp(-g))).to(torch.bfloat16).float()
    h_ref = (s * u).to(torch.bfloat16).float()
    check(blk.h[:P], h_ref, "swiglu")
    check(blk.y_seg[:P], y_ref, "down")
    if "zipf" in case and case["T"] > 384:
        assert max(cnt) > 384

    # backward: dh = dcur @ W_dn[e] with SwiGLU backward fused; dx = dgu @ W_gu[e]
    H = case["H"]
    g2 = torch.Generator(device=dev).manual_seed(7)
    blk.dcur[:P] = torch.randn(P, H, device=dev, generator=g2).to(torch.bfloat16)
    _lib.call("usaf_expert_down_bwd", blk.plan, p["down_proj"].struct(), _lib.ptr(blk.dcur),
              _lib.ptr(blk.gu), _lib.BF16, _lib.ptr(blk.dgu), st)
    _lib.call("usaf_expert_gate_up_bwd", blk.plan, p["gate_up_proj"].struct(), _lib.ptr(blk.dgu),
              _lib.BF16, _lib.ptr(blk.dx_seg), st)
    torch.cuda.synchronize()
    blk.check()
    dh_ref = torch.empty(P, I, device=dev)
    for e in range(case["E"]):
        if cnt[e]:
            sl = slice(off[e], off[e] + cnt[e])
            dh_ref[sl] = (blk.dcur[sl].float() @ wdn[e]).to(torch.bfloat16).float()
    sg = (g / (1 + torch.exp(-g))).to(torch.bfloat16).float()
    ds = (dh_ref * u).to(torch.bfloat16).float()
    du_ref = (dh_ref * sg).to(torch.bfloat16).float()
    sig = 1 / (1 + torch.exp(-g))
    dg_ref = (ds * sig * (1 + g * (1 - sig))).to(torch.bfloat16).float()
    check(blk.dgu[:P, I:], du_ref, "down_bwd/du")
    # dg goes through two bf16-rounded intermediates (dh, ds) that may each land
    # one step away from the reference's: 4 ulps
    check(blk.dgu[:P, :I], dg_ref, "down_bwd/dg", ulps=4)
    dx_ref = torch.empty(P, H, device=dev)
    for e in range(case["E"]):
        if cnt[e]:
            sl = slice(off[e], off[e] + cnt[e])
            dx_ref[sl] = (blk.dgu[sl].float() @ wgu[e]).to(torch.bfloat16).float()
    check(blk.dx_seg[:P], dx_ref, "gate_up_bwd")


@pytest.mark.parametrize("ci", [2, 4, 5], ids=["T2048_zipf", "T256_skew", "T4096_zipf"])
def test_grouped_gemms_write_every_item_repeatably(dev, ci):
    """Every launch writes every output of every work item, and repeated
    launches give bit-identical results: the work items are handed out at run
    time (longest first, to whichever CTA asks next), so a ticket must name
    the same item in every CTA and no item may be dropped or done twice with
    different inputs.  Outputs are filled with NaN before each launch."""
    from usaf_b200 import _lib
    case = CASES[ci]
    blk, x, w_r, p = make_case(dev, **case)
    st = _lib.stream()
    _lib.call("usaf_router_fwd", _lib.ptr(x), _lib.ptr(w_r), _lib.BF16, case["T"], case["H"],
              case["E"], case["k"], 1, _lib.ptr(blk.logits), _lib.ptr(blk.probs),
              _lib.ptr(blk.wsum), _lib.ptr(blk.weights), _lib.ptr(blk.router_ws), _lib.ptr(blk.err), st)
    _lib.call("usaf_dispatch", blk.plan, _lib.ptr(blk.weights), _lib.ptr(x), _lib.BF16, case["H"],
              _lib.ptr(blk.x_perm), st)
    torch.cuda.synchronize()
    P = blk.n_pairs_host()
    g2 = torch.Generator(device=dev).manual_seed(7)
    blk.dcur[:P] = torch.randn(P, case["H"], device=dev, generator=g2).to(torch.bfloat16)
    first = None
    for _ in range(30):
        outs = (blk.gu, blk.h, blk.y_seg, blk.dgu, blk.dx_seg)
        for t in outs:
            t.fill_(float("nan"))
        _lib.call("usaf_expert_gate_up_fwd", blk.plan, p["gate_up_proj"].struct(), _lib.ptr(blk.x_perm),
                  _lib.BF16, _lib.ptr(blk.gu), _lib.ptr(blk.h), st)
        _lib.call("usaf_expert_down_fwd", blk.plan, p["down_proj"].struct(), _lib.ptr(blk.h), _lib.BF16,
                  _lib.ptr(blk.y_seg), st)
        _lib.call("usaf_expert_down_bwd", blk.plan, p["down_proj"].struct(), _lib.ptr(blk.dcur),
                  _lib.ptr(blk.gu), _lib.BF16, _lib.ptr(blk.dgu), st)
        _lib.call("usaf_expert_gate_up_bwd", blk.plan, p["gate_up_proj"].struct(), _lib.ptr(blk.dgu),
                  _lib.BF16, _lib.ptr(blk.dx_seg), st)
        torch.cuda.synchronize()
        blk.check()
        got = [t[:P].clone() for t in outs]
        for name, t in zip(("gu", "h", "y", "dgu", "dx"), got):
            assert not torch.isnan(t.float()).any(), f"{name}: outputs left unwritten"
        if first is None:
            first = got
        for name, a, b in zip(("gu", "h", "y", "dgu", "dx"), got, first):
            assert torch.equal(a, b), f"{name}: launches differ"
    # the work counters are back at zero for the next launch
    assert int(blk.sched.abs().sum()) == 0


@pytest.mark.parametrize("ci", [3, 4], ids=["T512_C2", "T256_skew"])
def test_in_kernel_dequant_bit_exact(dev, ci):
    """With one-hot activation rows the grouped GEMMs return single weights:
    gu[s, r] = W_gu[e][r][c(s)] (forward) and dx[s, c] = W_gu[e][r(s)][c]
    (transposed backward), each one product 1 * w accumulated in fp32, so
    the kernels' in-register dequant and overlay patch must equal the
    reference's bf16(fp16(fp16(q*s)+z)) with trained values
    (usaf/quantization.py:59-79, usaf/moe_loader.py:241-247) bit for bit."""
    from usaf_b200 import _lib
    case = CASES[ci]
    blk, x, w_r, p = make_case(dev, **case)
    st = _lib.stream()
    _lib.call("usaf_router_fwd", _lib.ptr(x), _lib.ptr(w_r), _lib.BF16, case["T"], case["H"],
              case["E"], case["k"], 1, _lib.ptr(blk.logits), _lib.ptr(blk.probs),
              _lib.ptr(blk.wsum), _lib.ptr(blk.weights), _lib.ptr(blk.router_ws), _lib.ptr(blk.err), st)
    _lib.call("usaf_dispatch", blk.plan, _lib.ptr(blk.weights), _lib.ptr(x), _lib.BF16, case["H"],
              _lib.ptr(blk.x_perm), st)
    torch.cuda.synchronize()
    P = blk.n_pairs_host()
    H, I = case["H"], case["I"]
    off = blk.expert_off.cpu().tolist()
    cnt = blk.expert_cnt.cpu().tolist()
    exp_of = torch.repeat_interleave(torch.arange(case["E"], device=dev),
                                     torch.tensor(cnt, device=dev), output_size=P)
    s_idx = torch.arange(P, device=dev)
    wgu = eff_weight(p["gate_up_proj"]).to(torch.bfloat16)          # [E, 2I, H]
    # forward: slot s reads input column c(s)
    c_of = (s_idx * 37) % H
    blk.x_perm[:P].zero_()
    blk.x_perm[s_idx, c_of] = 1.0
    _lib.call("usaf_expert_gate_up_fwd", blk.plan, p["gate_up_proj"].struct(), _lib.ptr(blk.x_perm),
              _lib.BF16, _lib.ptr(blk.gu), _lib.ptr(blk.h), st)
    # transposed backward: slot s reads weight row r(s)
    r_of = (s_idx * 29) % (2 * I)
    blk.dgu[:P].zero_()
    blk.dgu[s_idx, r_of] = 1.0
    _lib.call("usaf_expert_gate_up_bwd", blk.plan, p["gate_up_proj"].struct(), _lib.ptr(blk.dgu),
              _lib.BF16, _lib.ptr(blk.dx_seg), st)
    torch.cuda.synchronize()
    blk.check()
    want_fwd = wgu[exp_of, :, c_of]                                   # [P, 2I]
    assert torch.equal(blk.gu[:P], want_fwd), \
        f"forward: {int((blk.gu[:P] != want_fwd).sum())} weights differ"
    want_bwd = wgu[exp_of, r_of, :]                                   # [P, H]
    assert torch.equal(blk.dx_seg[:P], want_bwd), \
        f"transposed: {int((blk.dx_seg[:P] != want_bwd).sum())} weights differ"
    assert off[-1] == P

