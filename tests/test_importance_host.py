"""ImportanceScorer host logic (usaf/importance.py:24-111) on a small dense
CPU model: skip patterns, |grad| sums over batches, max_batches, 1-D
inputs, the out-of-memory skip rule, frozen parameters afterwards, and the
fp16 score file."""
import types

import pytest
import torch

from usaf_b200.importance import ImportanceScorer


class Tiny(torch.nn.Module):
    def __init__(self):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        self.embed_tokens = torch.nn.Embedding(16, 8)
        self.body = torch.nn.Linear(8, 8)
        self.lm_head = torch.nn.Linear(8, 16, bias=False)
        for p in self.parameters():
            p.data = torch.randn(p.shape, generator=g)
        self.fail = None
        self.calls = 0

    def forward(self, input_ids, labels):
        self.calls += 1
        if self.fail is not None and self.calls in self.fail:
            raise RuntimeError(self.fail[self.calls])
        h = torch.tanh(self.body(self.embed_tokens(input_ids)))
        logits = self.lm_head(h)
        loss = torch.nn.functional.cross_entropy(logits.reshape(-1, 16), labels.reshape(-1))
        return types.SimpleNamespace(loss=loss)


def batches(n, seed=1):
    g = torch.Generator().manual_seed(seed)
    out = []
    for _ in range(n):
        ids = torch.randint(0, 16, (2, 5), generator=g)
        out.append({"input_ids": ids, "labels": ids})
    return out


def manual(model, bs):
    acc = {}
    for b in bs:
        model.zero_grad(set_to_none=True)
        model(b["input_ids"], b["labels"]).loss.backward()
        for n in ("body.weight", "body.bias"):
            g = getattr(model, n.split(".")[0]).__getattr__(n.split(".")[1]).grad.abs()
            acc[n] = acc[n] + g if n in acc else g
    return acc


def test_sums_skip_and_freeze():
    m = Tiny()
    bs = batches(3)
    for p in m.parameters():
        p.requires_grad_(True)
    ref = manual(m, bs)
    sc = ImportanceScorer(m, torch.device("cpu"), torch.float32).compute_scores(bs)
    for n in ref:
        assert torch.allclose(sc[n], ref[n], rtol=1e-6, atol=0), n
    assert sc["embed_tokens.weight"].abs().sum() == 0 and sc["lm_head.weight"].abs().sum() == 0
    assert all(not p.requires_grad for p in m.parameters())
    assert set(sc) == {n for n, _ in m.named_parameters()}


def test_max_batches_and_1d():
    m = Tiny()
    bs = batches(3)
    one = ImportanceScorer(m, torch.device("cpu"), torch.float32).compute_scores(bs, max_batches=1)
    m2 = Tiny()
    for p in m2.parameters():
        p.requires_grad_(True)
    ref = manual(m2, bs[:1])
    assert torch.allclose(one["body.weight"], ref["body.weight"], rtol=1e-6, atol=0)
    flat = [{"input_ids": b["input_ids"][0], "labels": b["labels"][0]} for b in bs[:1]]
    m3 = Tiny()
    sc = ImportanceScorer(m3, torch.device("cpu"), torch.float32).compute_scores(flat)
    assert sc["body.weight"].abs().sum() > 0


def test_oom_skip_and_other_errors():
    m = Tiny()
    m.fail = {1: "CUDA out of memory. Tried to allocate 2 GiB"}
    bs = batches(2)
    sc = ImportanceScorer(m, torch.device("cpu"), torch.float32).compute_scores(bs)
    m2 = Tiny()
    for p in m2.parameters():
        p.requires_grad_(True)
    ref = manual(m2, bs[1:])
    assert torch.allclose(sc["body.weight"], ref["body.weight"], rtol=1e-6, atol=0)
    m = Tiny()
    m.fail = {1: "shape mismatch"}
    with pytest.raises(RuntimeError, match="shape mismatch"):
        ImportanceScorer(m, torch.device("cpu"), torch.float32).compute_scores(bs)
    assert all(not p.requires_grad for p in m.parameters())


def test_score_file(tmp_path):
    m = Tiny()
    s = ImportanceScorer(m, torch.device("cpu"), torch.float32)
    sc = s.compute_scores(batches(1))
    s.save_scores(sc, str(tmp_path / "s.pt"))
    back = ImportanceScorer.load_scores(str(tmp_path / "s.pt"))
    assert back["body.weight"].dtype == torch.float16
    assert torch.equal(back["body.weight"], sc["body.weight"].half())
