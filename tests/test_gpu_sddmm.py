"""Expert-weight gradients at the selected coordinates (usaf_sparse_dw) and the
dense |gradient| of the importance pass (usaf_expert_dense_dw) on the
tensor-core path, against a plain torch fp32 reference of the same op:
per expert segment D_e = gout_e^T gin_e in fp32, rounded to bf16, gathered at
the overlay coordinates in compact order and scaled.

Tolerance: both sides accumulate in fp32 in different orders before the
bf16 rounding, so a value may land one bf16 step away: |diff| <= 1 bf16 ulp
of the reference (at most 2^-7 of its magnitude) + 1e-6 absolute, relative Frobenius error
<= 4e-3.  The SIMT kernel (selected by a NULL overlay bitmap) is held to the
same bound against the same reference.
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


def skewed_selection(numel, R, C, frac, g, dev):
    """Half the coordinates packed into a few heavy rows, the rest uniform."""
    n = max(2, int(numel * frac))
    heavy_rows = torch.randint(0, numel // C, (4,), device=dev, generator=g)
    cols = torch.randperm(C, device=dev, generator=g)[: min(C, n // 8)]
    heavy = (heavy_rows[:, None] * C + cols[None, :]).reshape(-1)
    rest = torch.randperm(numel, device=dev, generator=g)[:n]
    idx = torch.unique(torch.cat([heavy, rest]))
    return idx[torch.randperm(idx.numel(), device=dev, generator=g)]   # compact order is arbitrary


def build(dev, T, H, E, k, I, zipf, seed, skew):
    from usaf_b200.engine import BlockDims, MoEBlock, Projection
    from usaf_b200.quantization import quantize_4bit
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    w_r = torch.randn(E, H, device=dev, generator=g) * 0.02
    x[:, 0] = 1.0
    p = torch.arange(1, E + 1, device=dev, dtype=torch.float64) ** (-zipf)
    w_r[:, 0] += torch.log(p / p.sum()).float()          # skewed routing: some experts get no slots
    w_r = w_r.to(torch.bfloat16)
    dy = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    projs = {}
    for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = torch.randn(*shape, device=dev, generator=g) * 0.02
        q, s, z, _ = quantize_4bit(w, 128)
        pr = Projection(q, s, z, shape, 128, torch.bfloat16)
        numel = pr.numel()
        if skew:
            idx = skewed_selection(numel, shape[1], shape[2], 0.005, g, dev)
        else:
            idx = torch.randperm(numel, device=dev, generator=g)[: int(numel * 0.005)]
        pr.set_overlay(idx, torch.randn(idx.numel(), device=dev, generator=g) * 0.02)
        pr.idx = idx
        projs[n] = pr
    blk = MoEBlock(BlockDims(T, H, E, I, k, True, torch.bfloat16), dev)
    blk.forward(x, w_r, projs["gate_up_proj"], projs["down_proj"])
    blk.backward(dy, x, w_r, projs["gate_up_proj"], projs["down_proj"])
    torch.cuda.synchronize()
    blk.check()
    return blk, projs


def dense_ref(blk, gout, gin, R, C):
    off = blk.expert_off.cpu().tolist()
    E = len(off) - 1
    D = torch.zeros(E, R, C, dtype=torch.float32, device=gout.device)
    for e in range(E):
        a, b = off[e], off[e + 1]
        if b > a:
            D[e] = gout[a:b].float().t() @ gin[a:b].float()
    return D.to(torch.bfloat16).float()


def check(got, ref, what):
    tol = ref.abs() * 2 ** -7 + 1e-6
    bad = (got - ref).abs() > tol
    rel = ((got - ref).norm() / ref.norm().clamp_min(1e-30)).item()
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.numel()} beyond 1 bf16 ulp; rel {rel:.2e}"
    assert rel <= 4e-3, f"{what}: rel {rel:.2e}"


CASES = [
    # the first three run the tensor-core kernel (pair capacity above 64 per expert)
    dict(T=320, H=512, E=32, k=4, I=384, zipf=1.5, seed=3, skew=True),     # C % 256 == 128 tiles
    dict(T=320, H=512, E=16, k=2, I=256, zipf=0.0, seed=4, skew=False),    # experts of ~40 slots (< 64)
    dict(T=1024, H=2048, E=128, k=8, I=768, zipf=1.2, seed=5, skew=True),  # Qwen3-30B-A3B shapes
    dict(T=8, H=512, E=32, k=4, I=384, zipf=0.0, seed=6, skew=True),       # decode-sized: CUDA-core path
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: "T{T}_H{H}_E{E}_I{I}".format(**c) + ("_skew" if c["skew"] else ""))
def test_sparse_dw_tc_vs_torch(dev, case):
    from usaf_b200 import _lib
    blk, projs = build(dev, **case)
    operands = {"gate_up_proj": (blk.dgu, blk.x_perm), "down_proj": (blk.dcur, blk.h)}
    st = _lib.stream()
    scale = 0.5
    for n, p in projs.items():
        assert p.ov_mask is not None
        gout, gin = operands[n]
        ref = scale * dense_ref(blk, gout, gin, p.R, p.C).reshape(-1)[p.idx]
        got = torch.zeros(p.n_ov, dtype=torch.float32, device=dev)
        _lib.call("usaf_sparse_dw", blk.plan, p.struct(), _lib.ptr(gout), _lib.ptr(gin), _lib.BF16,
                  _lib.ptr(p.csr_to_compact), scale, _lib.ptr(got), _lib.ptr(p.scratch), st)
        simt = torch.zeros_like(got)
        s2 = _lib.QWeight.from_buffer_copy(p.struct())
        s2.ov_mask = None                      # NULL bitmap: the SIMT kernel
        _lib.call("usaf_sparse_dw", blk.plan, s2, _lib.ptr(gout), _lib.ptr(gin), _lib.BF16,
                  _lib.ptr(p.csr_to_compact), scale, _lib.ptr(simt), _lib.ptr(p.scratch), st)
        torch.cuda.synchronize()
        blk.check()
        check(got, ref, f"{n} tensor-core")
        check(simt, ref, f"{n} simt")


@pytest.mark.parametrize("case", CASES[:2], ids=lambda c: "T{T}_H{H}_E{E}_I{I}")
def test_dense_abs_dw_tc_vs_torch(dev, case):
    from usaf_b200 import _lib
    blk, projs = build(dev, **case)
    operands = {"gate_up_proj": (blk.dgu, blk.x_perm), "down_proj": (blk.dcur, blk.h)}
    st = _lib.stream()
    for n, p in projs.items():
        gout, gin = operands[n]
        ref = dense_ref(blk, gout, gin, p.R, p.C).abs()
        got = torch.full((p.E, p.R, p.C), float("nan"), dtype=torch.float32, device=dev)
        _lib.call("usaf_expert_dense_dw", blk.plan, p.R, p.C, _lib.ptr(gout), _lib.ptr(gin), _lib.BF16,
                  _lib.ptr(got), st)
        torch.cuda.synchronize()
        blk.check()
        assert not got.isnan().any(), f"{n}: coordinates left unwritten"
        check(got, ref, f"{n} dense |dW|")
