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


def _fixture_case(golden_dir, fname):
    """Inputs of one tensor of the reference-generated RigL fixture; the int4
    entry is the C1 dequant re-quantized (checked against the fixture's hash)."""
    import os
    import numpy as np
    from oracle import quant as oquant
    from oracle.inputs import C1, make_block_inputs
    import hashlib

    def sha(*arrays):
        h = hashlib.sha256()
        for a in arrays:
            h.update(np.ascontiguousarray(a).tobytes())
        return h.hexdigest()
    g = torch.load(os.path.join(golden_dir, "rigl.pt"), weights_only=False)
    inp = make_block_inputs(**C1)
    src = "gate_up_proj" if fname.endswith("gate_up_proj") else "down_proj"
    q, s, z, shape = oquant.quantize_4bit(inp[src]["fp16"].astype(np.float32), 128)
    assert sha(q, s, z) == g[f"{fname}.qsz_sha"]
    orig = torch.from_numpy(oquant.dequantize_4bit(q, s, z, shape, 128)).reshape(-1)
    return g, orig


@pytest.mark.parametrize("fname", ["t.gate_up_proj", "t.down_proj", "t.keep"])
def test_merge_vs_reference_fixture(dev, golden_dir, fname):
    """usaf_b200.rigl.merge against the reference's own merge loop
    (train.py:552-596, run by tests/golden/make_golden.py): identical final
    index list (kept then grown, each ascending) and identical values."""
    from usaf_b200 import rigl
    g, orig = _fixture_case(golden_dir, fname)
    new = g[f"{fname}.new"]
    got_idx, got_vals = rigl.merge(g[f"{fname}.old"].to(dev), None if new is None else new.to(dev),
                                   g[f"{fname}.masters"].to(dev), orig.to(dev))
    assert torch.equal(got_idx.cpu().long(), g[f"{fname}.final"].long())
    assert torch.equal(got_vals.cpu().float(), g[f"{fname}.final_masters"])
