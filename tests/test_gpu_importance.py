"""Importance candidates without the dense |grad| buffer.

The fused path (three tensor-core SDDMM passes: exponent histogram,
histogram inside the threshold bucket, emission; then device sorts) must
give every expert exactly the candidate list of the dense path it replaces:
the dense |dtype(dW_e)| of usaf_expert_dense_dw followed by usaf_topk_desc
(top k = max(1, int(numel_e * frac * 2)), descending, equal scores by
ascending flat index; usaf/moe_loader.py:604-611).  Bit-identical values and
indices, same experts (those with routed slots), including experts whose
slots span several SDDMM chunks and thresholds that fall on ties."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import usaf_b200  # noqa: F401
    return torch.device("cuda:0")


def _layer(dev, T, H, E, k, I, zipf=None, zero_cols=None, seed=0):
    from usaf_b200.engine import Projection
    from usaf_b200.layer import SparseMoELayer
    from usaf_b200.quantization import quantize_4bit
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, H, device=dev, generator=g)
    w_r = torch.randn(E, H, device=dev, generator=g) * 0.02
    if zipf is not None:
        x[:, 0] = 1.0
        p = torch.arange(1, E + 1, device=dev, dtype=torch.float64) ** (-zipf)
        w_r[:, 0] += torch.log(p / p.sum()).float()
    if zero_cols is not None:
        x[:, zero_cols:] = 0.0        # gate_up gradient columns past zero_cols are exactly zero
    x = x.to(torch.bfloat16)
    w_r = w_r.to(torch.bfloat16)
    projs = {}
    for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = torch.randn(*shape, device=dev, generator=g) * 0.02
        q, s, z, _ = quantize_4bit(w, 128)
        projs[n] = Projection(q, s, z, shape, 128, torch.bfloat16)
    dy = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    layer = SparseMoELayer(w_r, projs["gate_up_proj"], projs["down_proj"], k, T)
    layer.forward_backward(x, dy)
    torch.cuda.synchronize()
    layer.block.check()
    return layer


CASES = {
    "C2_T512": dict(T=512, H=2048, E=128, k=8, I=768),
    "C2_T4096_zipf": dict(T=4096, H=2048, E=128, k=8, I=768, zipf=1.2),   # experts > 320 slots
    "ties_at_zero": dict(T=256, H=512, E=16, k=4, I=256, zero_cols=2),     # threshold on zeros
    "tiny_C128": dict(T=64, H=256, E=8, k=2, I=128),                        # 128-column tiles (down)
}


@pytest.mark.parametrize("name", list(CASES))
def test_fused_candidates_equal_dense_path(dev, name):
    from usaf_b200 import _lib, engine
    layer = _layer(dev, **CASES[name])
    blk = layer.block
    cnt = blk.expert_cnt.cpu()
    if name == "C2_T4096_zipf":
        assert int(cnt.max()) > int(_lib.LIB.usaf_importance_chunk_slots())
    for which in ("gate_up_proj", "down_proj"):
        p = layer.gu if which == "gate_up_proj" else layer.dn
        numel_e = p.R * p.C
        kk = min(max(1, int(numel_e * 0.005 * 2.0)), numel_e)
        got = blk.expert_candidates(which, kk)
        assert got is not None
        vals, idx, experts = got
        assert experts.tolist() == (cnt > 0).nonzero().reshape(-1).tolist()
        dense = blk.dense_abs_grad(which)
        n_tie_rows = 0
        for row, e in enumerate(experts.tolist()):
            rv, ri = engine.topk_desc(dense[e].reshape(-1), kk, idx_base=e * numel_e)
            n_tie_rows += int((rv == rv[-1]).sum() > 1)
            order = torch.argsort(ri)                    # fused rows are in index order
            rv, ri = rv[order], ri[order]
            gv, gi = vals[row * kk:(row + 1) * kk], idx[row * kk:(row + 1) * kk]
            assert torch.equal(gi, ri), f"{which} expert {e}: indices differ"
            assert torch.equal(gv, rv), f"{which} expert {e}: values differ"
        if name == "ties_at_zero" and which == "gate_up_proj":
            # the case is built so that some list ends inside a run of equal scores
            assert n_tie_rows > 0


def test_store_selection_fused_vs_dense(dev):
    """TopKImportanceStore.add_from (fused) and add_dense_abs (dense) give the
    same per-tensor selection (usaf/moe_loader.py:613-628) and the same
    per-expert lists from candidates() (descending score, ties by index)."""
    from usaf_b200.moe_loader import TopKImportanceStore
    layer = _layer(dev, **CASES["C2_T512"])
    blk = layer.block
    a = TopKImportanceStore(layer.shapes, 0.005)
    b = TopKImportanceStore(layer.shapes, 0.005)
    for name in layer.names:
        which = name.rsplit(".", 1)[1]
        a.add_from(name, blk, which)
        b.add_dense_abs(name, blk.dense_abs_grad(which), blk.hit_experts())
    sa, sb = a.select(), b.select()
    for name in sa:
        assert torch.equal(sa[name], sb[name]), name
        va, ia = a.candidates(name)
        vb, ib = b.candidates(name)
        assert sorted(va) == sorted(vb)
        for e in va:
            assert torch.equal(va[e], vb[e]) and torch.equal(ia[e], ib[e]), (name, e)
