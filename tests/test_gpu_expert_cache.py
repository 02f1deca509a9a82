"""QuantizedExpertCache (usaf_b200.moe_loader, drop-in for
usaf/moe_loader.py:60-524): q4 entries in both of the reference's forms (dict
and 4-tuple, train.py:175-177) become resident projections;
apply_resident_overlays installs trained coordinates and sync_resident
refreshes their values after the masters change (usaf/moe_loader.py:
226-247, 411-443).  Checked through the grouped GEMMs: the experts' output
equals torch fp32 on the effective weights (fp16 dequant with fp16(master)
at the trained coordinates), before and after the masters move.

Tolerance: bf16 outputs within 2 bf16 ulp (+1e-3 absolute) and relative
Frobenius error <= 4e-3 (the GEMM tests' bound)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

E, K, H, I, T = 4, 2, 256, 128, 64


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import usaf_b200  # noqa: F401
    return torch.device("cuda:0")


def _check(got, ref):
    got, ref = got.float(), ref.float()
    assert not ((got - ref).abs() > ref.abs() * 2 ** -7 * 2 + 1e-3).any()
    assert ((got - ref).norm() / ref.norm()).item() <= 4e-3


def _experts_ref(x, weights, w_gu, w_dn):
    y = torch.zeros(x.shape, dtype=torch.float32, device=x.device)
    for e in range(E):
        tok = (weights[:, e] != 0).nonzero().reshape(-1)
        if tok.numel() == 0:
            continue
        gu = (x[tok].float() @ w_gu[e].T).to(torch.bfloat16).float()
        g, u = gu[:, :I], gu[:, I:]
        h = ((g / (1 + torch.exp(-g))).to(torch.bfloat16).float() * u).to(torch.bfloat16).float()
        yd = (h @ w_dn[e].T).to(torch.bfloat16).float()
        y[tok] += yd * weights[tok, e].float()[:, None]
    return y.to(torch.bfloat16)


def test_cache_overlays_and_sync(dev):
    from usaf_b200.engine import BlockDims, MoEBlock
    from usaf_b200.moe_loader import QuantizedExpertCache
    from usaf_b200.quantization import quantize_4bit
    g = torch.Generator(device=dev).manual_seed(4)
    q_dict, shapes = {}, {}
    for i, (which, shape) in enumerate((("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I)))):
        q, s, z, sh = quantize_4bit(torch.randn(*shape, device=dev, generator=g) * 0.02, 128)
        name = f"layer.mlp.experts.{which}"
        # one entry as the reference's dict, the other as its 4-tuple
        q_dict[name] = ({"q": q.cpu(), "s": s.cpu(), "z": z.cpu(), "shape": tuple(sh)} if i == 0
                        else (q.cpu(), s.cpu(), z.cpu(), tuple(sh)))
        shapes[name] = shape
    cache = QuantizedExpertCache(q_dict, dev)
    assert set(cache.projections) == set(q_dict)
    active = {n: torch.randperm(torch.Size(sh).numel(), device=dev, generator=g)[:2000] for n, sh in shapes.items()}
    masters = {n: cache.dequant(n).reshape(-1)[active[n]].float() + 0.01 for n in shapes}
    cache.apply_resident_overlays(active, masters)
    assert all(cache.overlays[n][0] is active[n] for n in shapes)
    gu, dn = cache.projection("layer.mlp.experts.gate_up_proj"), cache.projection("layer.mlp.experts.down_proj")
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, device=dev, generator=g)
    top = logits.topk(K, dim=1)
    weights = torch.zeros(T, E, device=dev).scatter_(1, top.indices, top.values.softmax(1)).to(torch.bfloat16)
    blk = MoEBlock(BlockDims(T, H, E, I, K, True, torch.bfloat16), dev)

    def effective(n):
        w = cache.dequant(n).reshape(-1).clone()
        w[active[n]] = masters[n].half()
        return w.view(shapes[n]).to(torch.bfloat16).float()

    for rnd in range(2):
        y = blk.experts_forward(x, weights, gu, dn).clone()
        torch.cuda.synchronize()
        blk.check()
        _check(y, _experts_ref(x, weights, effective("layer.mlp.experts.gate_up_proj"),
                               effective("layer.mlp.experts.down_proj")))
        # the masters move; sync_resident pushes them into the resident overlay
        for n in masters:
            masters[n] += 0.05 * torch.randn(masters[n].shape, device=dev, generator=g)
        cache.sync_resident(active, masters)
