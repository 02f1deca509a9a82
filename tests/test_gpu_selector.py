"""Device selectors (usaf_b200.selector) against the reference's own selector
tests (tests/test_selector.py:13-63 of the reference, same inputs on the
device) and against the oracle restatement (oracle/moe.py, numpy partition)
on large tensors with many ties.  Masks must be identical (bit-exact)."""
import pytest
import torch

from oracle import moe as omoe

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import usaf_b200  # noqa: F401
    return torch.device("cuda:0")


def test_reference_cases(dev):
    from usaf_b200.selector import DynamicSelector, ThresholdSelector, TopKSelector
    assert TopKSelector(k=100).select({}) == {}
    s = {"layer1.weight": torch.tensor([1.0, 2.0, 3.0, 4.0, 5.0], device=dev),
         "layer2.weight": torch.tensor([0.1, 0.2, 0.3], device=dev)}
    assert sum(int(m.sum()) for m in TopKSelector(k=3).select(s).values()) == 3
    assert int(TopKSelector(k=10).select({"w1": torch.tensor([1.0, 2.0, 3.0], device=dev)})["w1"].sum()) == 3
    m = ThresholdSelector(percentile=50.0).select({"w1": torch.tensor([0.1, 0.5, 0.9, 1.0], device=dev)})["w1"]
    assert m.cpu().tolist() == [False, False, True, True]
    sel = DynamicSelector(initial_k=2, reselect_every_n_steps=10)
    assert sel.active_mask == {}
    mask = sel.update_mask({"w1": torch.tensor([1.0, 2.0, 3.0, 4.0, 5.0], device=dev)}, k=2)
    assert int(mask["w1"].sum()) == 2 and len(sel.active_mask) == 1


@pytest.mark.parametrize("k", [1, 7, 1000, 123457, 10 ** 9])
def test_topk_vs_oracle_with_ties(dev, k):
    from usaf_b200.selector import TopKSelector
    g = torch.Generator().manual_seed(k % 1000)
    # quantised scores -> heavy ties; a few zeros and denormal-size values
    scores = {f"t{i}": (torch.randint(0, 500, (n,), generator=g).float() * 1e-3)
              for i, n in enumerate((300_000, 1_000_003, 77))}
    scores["t0"][:10] = 0.0
    ref = omoe.topk_select(scores, k)
    got = TopKSelector(k).select({n: s.to(dev) for n, s in scores.items()})
    for n in scores:
        assert torch.equal(got[n].cpu(), ref[n]), n


@pytest.mark.parametrize("pct", [0.0, 50.0, 99.98, 100.0])
def test_threshold_vs_oracle(dev, pct):
    from usaf_b200.selector import ThresholdSelector
    g = torch.Generator().manual_seed(3)
    scores = {"a": torch.rand(400_001, generator=g), "b": torch.randn(5000, generator=g).abs()}
    ref = omoe.threshold_select(scores, pct)
    got = ThresholdSelector(pct).select({n: s.to(dev) for n, s in scores.items()})
    for n in scores:
        assert torch.equal(got[n].cpu(), ref[n]), n
