"""The allocation-free entry point usaf_sparse_dw_noalloc.

Callers that cannot allocate device memory when they call in (a process that
works inside a memory pool reserved at start-up, or a foreign-language host
that can only hand over buffers it already owns) use this variant: its
per-coordinate scratch is a fixed array inside the library instead of a
buffer the caller passes.  It must produce what usaf_sparse_dw produces with
a caller-provided scratch buffer, call after call (the shared array keeps the
previous call's contents).  Collected last on purpose (file name).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = 1e-6  # relative; the kernel is deterministic, so the results are equal


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import usaf_b200  # noqa: F401
    return torch.device("cuda:0")


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


# T=512: the tensor-core kernel; T=64: at most 64 pair slots per expert
# (P_cap = 64 * 8 = 512 <= 64 * E), the CUDA-core kernel
@pytest.mark.parametrize("T", [512, 64])
def test_noalloc_matches_scratch_entry_point(dev, T):
    from usaf_b200 import _lib
    from usaf_b200.engine import BlockDims, MoEBlock, Projection
    from usaf_b200.quantization import quantize_4bit
    H, E, k, I = 512, 16, 4, 256
    g = torch.Generator(device=dev).manual_seed(11)
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    dy = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    w_r = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    proj = {}
    for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = torch.randn(*shape, device=dev, generator=g) * 0.02
        q, s, z, _ = quantize_4bit(w, 128)
        p = Projection(q, s, z, shape, 128, torch.bfloat16)
        idx = torch.randperm(p.numel(), device=dev, generator=g)[: int(p.numel() * 0.005)]
        p.set_overlay(idx, torch.randn(idx.numel(), device=dev, generator=g) * 0.02)
        proj[n] = p
    blk = MoEBlock(BlockDims(T, H, E, I, k, True, torch.bfloat16), dev)
    assert (blk.P_cap <= 64 * E) == (T == 64)
    blk.forward(x, w_r, proj["gate_up_proj"], proj["down_proj"])
    blk.backward(dy, x, w_r, proj["gate_up_proj"], proj["down_proj"])
    st = _lib.stream()
    operands = {"gate_up_proj": (blk.dgu, blk.x_perm), "down_proj": (blk.dcur, blk.h)}
    for n, p in proj.items():
        gout, gin = operands[n]
        ref = torch.zeros(p.n_ov, dtype=torch.float32, device=dev)
        got = torch.zeros(p.n_ov, dtype=torch.float32, device=dev)
        for call in range(2):  # two calls in a row: the compact vectors accumulate
            _lib.call("usaf_sparse_dw", blk.plan, p.struct(), _lib.ptr(gout), _lib.ptr(gin),
                      _lib.BF16, _lib.ptr(p.csr_to_compact), 1.0, _lib.ptr(ref), _lib.ptr(p.scratch), st)
            _lib.call("usaf_sparse_dw_noalloc", blk.plan, p.struct(), _lib.ptr(gout), _lib.ptr(gin),
                      _lib.BF16, _lib.ptr(p.csr_to_compact), 1.0, _lib.ptr(got), st)
            torch.cuda.synchronize()
            assert ref.abs().sum() > 0
            assert rel(got, ref) <= TOL, (n, call, rel(got, ref))
    blk.check()


def test_noalloc_rejects_oversized_overlay(dev):
    from usaf_b200 import _lib
    st = _lib.QWeight()
    st.E, st.R, st.C, st.group_size = 1, 2, 128, 128
    st.n_ov = (1 << 21) + 1   # one more coordinate than the built-in scratch holds
    plan = _lib.RoutePlan()
    with pytest.raises(_lib.UsafError, match="unsupported"):
        _lib.call("usaf_sparse_dw_noalloc", plan, st, 1, 1, _lib.BF16, 1, 1.0, 1, _lib.stream())
