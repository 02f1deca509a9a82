"""export_merged_weights on the device against the oracle restatement of
usaf/checkpoint.py:58-92 (numpy int4 dequantize, scatter fp16(master),
re-quantize): the exported q / s / z are bit-identical.  Also the
reference's own export test (tests/test_checkpoint.py:91-141)."""
import os

import numpy as np
import pytest
import torch

from oracle import quant as oquant

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import usaf_b200  # noqa: F401
    return torch.device("cuda:0")


def _oracle_export(qdict, masters, active, gs):
    out = {}
    for name, e in qdict.items():
        t = oquant.dequantize_4bit(e["q"].numpy(), e["s"].numpy(), e["z"].numpy(), e["shape"], gs)
        flat = np.array(t, dtype=np.float16).reshape(-1)
        if name in masters:
            flat[active[name].numpy()] = masters[name].numpy().astype(np.float16)
        q, s, z, shape = oquant.quantize_4bit(flat.reshape(e["shape"]).astype(np.float32), gs)
        out[name] = (q, s, z)
    return out


@pytest.mark.parametrize("gs", [4, 128])
def test_export_bit_exact_vs_oracle(dev, tmp_path, gs):
    from usaf_b200.checkpoint import export_merged_weights
    g = torch.Generator().manual_seed(gs)
    shapes = {"layer.mlp.experts.gate_up_proj": (4, 64, 256), "layer.mlp.experts.down_proj": (4, 256, 32)}
    qdict, masters, active = {}, {}, {}
    for name, shape in shapes.items():
        w = (torch.randn(*shape, generator=g) * 0.02).numpy()
        q, s, z, _ = oquant.quantize_4bit(w, gs)
        qdict[name] = {"q": torch.from_numpy(np.ascontiguousarray(q)), "s": torch.from_numpy(s),
                       "z": torch.from_numpy(z), "shape": torch.Size(shape), "group_size": gs}
        n = int(np.prod(shape))
        active[name] = torch.randperm(n, generator=g)[: n // 100]
        masters[name] = torch.randn(active[name].numel(), generator=g) * 0.05
    qpath = str(tmp_path / "orig_q4.pt")
    torch.save(qdict, qpath)
    out = str(tmp_path / "merged.pt")
    export_merged_weights(qpath, masters, active, out, group_size=gs)
    got = torch.load(out, weights_only=True)
    ref = _oracle_export(qdict, masters, active, gs)
    for name in shapes:
        q, s, z = ref[name]
        assert torch.equal(got[name]["q"], torch.from_numpy(np.ascontiguousarray(q))), name
        assert torch.equal(got[name]["s"], torch.from_numpy(s)), name
        assert torch.equal(got[name]["z"], torch.from_numpy(z)), name


def test_reference_export_case(dev, tmp_path):
    from usaf_b200.checkpoint import export_merged_weights
    from usaf_b200.quantization import dequantize_4bit, quantize_state_dict
    torch.manual_seed(0)
    orig = {"expert.w1": torch.randn(8, 8, dtype=torch.float16),
            "expert.w2": torch.randn(4, 4, dtype=torch.float16)}
    qd = {k: {kk: (vv.cpu() if isinstance(vv, torch.Tensor) else vv) for kk, vv in v.items()}
          for k, v in quantize_state_dict({k: v.to(dev) for k, v in orig.items()}, group_size=4, min_size=1).items()}
    qpath = str(tmp_path / "q.pt")
    torch.save(qd, qpath)
    masters = {"expert.w1": torch.tensor([99.0, 99.0]), "expert.w2": torch.tensor([88.0])}
    active = {"expert.w1": torch.tensor([0, 1]), "expert.w2": torch.tensor([3])}
    out = export_merged_weights(qpath, masters, active, str(tmp_path / "m.pt"), group_size=4)
    assert os.path.exists(out)
    merged = torch.load(out, weights_only=True)
    for name, t0 in orig.items():
        e = merged[name]
        if isinstance(e, dict):
            t = dequantize_4bit(e["q"].to(dev), e["s"].to(dev), e["z"].to(dev), e["shape"], 4).cpu().reshape(-1)
        else:   # below quantize_state_dict's min_size: kept as fp16
            t = e.reshape(-1).float()
        for i, idx in enumerate(active[name].tolist()):
            assert abs(t[idx].item() - masters[name][i].item()) < 0.1
