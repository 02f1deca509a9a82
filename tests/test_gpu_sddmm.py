"""Expert-weight gradients at the selected coordinates (usaf_sparse_dw) and the
dense |gradient| of the importance pass (usaf_expert_dense_dw) on the
tensor-core path, against a plain torch fp32 reference of the same op:
per expert segment D_e = gout_e^T gin_e in fp32, rounded to bf16, gathered at
the overlay coordinates in compact order and scaled.

Tolerance: both sides accumulate in fp32 in different orders before the
bf16 rounding (the tensor-core kernel also sums experts of more than 320
slots chunk by chunk), so a value may land one bf16 step away, and where the
slot products cancel the two fp32 sums differ by up to a few fp32 ulps of
the sum of their magnitudes S = sum_s |gout[s, r]| |gin[s, c]|:
|diff| <= 2^-7 |ref| + 2^-20 S + 1e-6, relative Frobenius error <= 4e-3.
The SIMT kernel (selected by a NULL overlay bitmap) is held to the same
bound against the same reference.
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


def dense_ref(blk, gout, gin, R, C, mag=False):
    """bf16(D_e) for every expert as fp32 [E, R, C]; with mag, also the sums of
    the products' magnitudes S_e = |gout_e|^T |gin_e|."""
    off = blk.expert_off.cpu().tolist()
    E = len(off) - 1
    D = torch.zeros(E, R, C, dtype=torch.float32, device=gout.device)
    S = torch.zeros_like(D) if mag else None
    for e in range(E):
        a, b = off[e], off[e + 1]
        if b > a:
            D[e] = gout[a:b].float().t() @ gin[a:b].float()
            if mag:
                S[e] = gout[a:b].float().abs().t() @ gin[a:b].float().abs()
    D = D.to(torch.bfloat16).float()
    return (D, S) if mag else D


def check(got, ref, what, mag=None):
    tol = ref.abs() * 2 ** -7 + 1e-6 + (mag * 2 ** -20 if mag is not None else 0.0)
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
    # experts of ~1000 slots on average: the streaming tensor-core kernel
    dict(T=4096, H=512, E=8, k=2, I=384, zipf=0.0, seed=7, skew=True),
    dict(T=4096, H=512, E=8, k=2, I=256, zipf=1.2, seed=8, skew=False),
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
        D, S = dense_ref(blk, gout, gin, p.R, p.C, mag=True)
        ref = scale * D.reshape(-1)[p.idx]
        mag = scale * S.reshape(-1)[p.idx]
        del D, S
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
        check(got, ref, f"{n} tensor-core", mag)
        check(simt, ref, f"{n} simt", mag)


@pytest.mark.parametrize("case", CASES[:3], ids=lambda c: "T{T}_H{H}_E{E}_I{I}")
def test_dense_abs_dw_tc_vs_torch(dev, case):
    from usaf_b200 import _lib
    blk, projs = build(dev, **case)
    operands = {"gate_up_proj": (blk.dgu, blk.x_perm), "down_proj": (blk.dcur, blk.h)}
    st = _lib.stream()
    for n, p in projs.items():
        gout, gin = operands[n]
        ref, mag = dense_ref(blk, gout, gin, p.R, p.C, mag=True)
        ref = ref.abs()
        got = torch.full((p.E, p.R, p.C), float("nan"), dtype=torch.float32, device=dev)
        _lib.call("usaf_expert_dense_dw", blk.plan, p.R, p.C, _lib.ptr(gout), _lib.ptr(gin), _lib.BF16,
                  _lib.ptr(got), st)
        torch.cuda.synchronize()
        blk.check()
        assert not got.isnan().any(), f"{n}: coordinates left unwritten"
        check(got, ref, f"{n} dense |dW|", mag)


@pytest.mark.parametrize("C", [128, 768, 2048])
def test_ov_cbptr_builder(dev, C):
    """usaf_build_ov_cbptr against a torch restatement: CSR position of the
    first entry of each (row, half) segment at or past every 256-column block."""
    from usaf_b200.engine import Projection
    from usaf_b200.quantization import quantize_4bit
    E, R = 3, 256
    g = torch.Generator(device=dev).manual_seed(C)
    q, s_, z, _ = quantize_4bit(torch.randn(E, R, C, device=dev, generator=g) * 0.02, 128)
    pr = Projection(q, s_, z, (E, R, C), 128, torch.bfloat16)
    n = E * R * C // 50
    idx = torch.randperm(E * R * C, device=dev, generator=g)[:n]
    heavy = torch.arange(C, device=dev) + 5 * C                      # one fully selected row
    idx = torch.unique(torch.cat([idx, heavy]))
    pr.set_overlay(idx, torch.zeros(idx.numel(), device=dev))
    torch.cuda.synchronize()
    ncb = (C + 255) // 256
    rows = torch.repeat_interleave(torch.arange(E * R * 2, device=dev), pr.row_ptr[1:].long() - pr.row_ptr[:-1].long())
    col = pr.col.long()
    expect = torch.empty(E * R, ncb, 2, dtype=torch.int64, device=dev)
    for b in range(ncb):
        below = torch.zeros(E * R * 2, dtype=torch.int64, device=dev)
        below.index_add_(0, rows, (col < 256 * b).long())
        expect[:, b, :] = (pr.row_ptr[:-1].long() + below).view(E * R, 2)
    assert torch.equal(pr.ov_cbptr.long().view(E * R, ncb, 2), expect)
