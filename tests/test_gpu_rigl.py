"""RigL reselection merge on the device (usaf_b200.rigl.merge) against the
oracle's restatement of train.py:552-596 (oracle/moe.py rigl_merge):
identical final index lists and identical carried / regrown values."""
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


CASES = ["overlap", "disjoint", "identical", "new_smaller", "new_larger", "none"]


@pytest.mark.parametrize("case", CASES)
def test_merge_vs_oracle(dev, case):
    from usaf_b200 import rigl
    g = torch.Generator().manual_seed(CASES.index(case))
    numel = 200_000
    orig = torch.randn(numel, generator=g).half()
    old = torch.randperm(numel, generator=g)[:5000]
    masters = torch.randn(old.numel(), generator=g)
    if case == "overlap":
        new = torch.cat([old[:2500], torch.randperm(numel, generator=g)[:4000]]).unique()
        new = new[torch.randperm(new.numel(), generator=g)]
    elif case == "disjoint":
        pool = torch.ones(numel, dtype=torch.bool)
        pool[old] = False
        cand = pool.nonzero().reshape(-1)
        new = cand[torch.randperm(cand.numel(), generator=g)[:5000]]
    elif case == "identical":
        new = old[torch.randperm(old.numel(), generator=g)]
    elif case == "new_smaller":
        new = torch.cat([old[:100], torch.randperm(numel, generator=g)[:1000]]).unique()
    elif case == "new_larger":
        new = torch.randperm(numel, generator=g)[:20000]
    else:
        new = None
    ref_idx, ref_vals = omoe.rigl_merge(old, new, masters, orig)
    got_idx, got_vals = rigl.merge(old.to(dev), None if new is None else new.to(dev),
                                   masters.to(dev), orig.to(dev))
    assert torch.equal(got_idx.cpu().long(), ref_idx.long())
    assert torch.equal(got_vals.cpu().float(), ref_vals.float())
