"""The step driver (usaf_b200.trainer.SparseTrainer) on a two-layer
Qwen3-MoE causal LM patched with patch_qwen3moe_for_b200 and int4 experts:

* importance selection, then steps with accumulation: losses finite, masters
  and router weights move, the SparseAdam state advances;
* a RigL reselection at the scheduled step keeps the per-tensor active count
  and restarts the optimizer state;
* a step with a non-finite loss is skipped (no master, moment or router
  change) and halves the loss scale;
* a checkpoint written by one trainer and loaded by another restores the
  active sets, masters, optimizer state and loss-scale state;
* ImportanceScorer scores the int4 experts through the capture protocol.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

E, K, H, I, LAYERS, VOCAB = 16, 4, 512, 256, 2, 512


@pytest.fixture(scope="module")
def model():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeForCausalLM
    from usaf_b200 import qwen3moe
    from usaf_b200.engine import Projection
    from usaf_b200.quantization import quantize_4bit
    qwen3moe.patch_qwen3moe_for_b200()
    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    cfg = Qwen3MoeConfig(vocab_size=VOCAB, hidden_size=H, intermediate_size=1024,
                         num_hidden_layers=LAYERS, num_attention_heads=4, num_key_value_heads=2,
                         head_dim=128, moe_intermediate_size=I, num_experts=E,
                         num_experts_per_tok=K, norm_topk_prob=True, max_position_embeddings=256)
    m = Qwen3MoeForCausalLM(cfg).to(device=dev, dtype=torch.bfloat16)
    for p in m.parameters():
        p.requires_grad_(False)
    g = torch.Generator(device=dev).manual_seed(1)
    for layer in m.model.layers:
        mlp = layer.mlp
        mlp.gate.weight.data = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        mlp.gate.weight.requires_grad_(True)
        projs = []
        for shape in ((E, 2 * I, H), (E, H, I)):
            w = torch.randn(*shape, device=dev, generator=g) * 0.02
            q, s, z, _ = quantize_4bit(w, 128)
            projs.append(Projection(q, s, z, shape, 128, torch.bfloat16))
        qwen3moe.attach_int4_experts(mlp.experts, *projs)
    return m


def _batches(n, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, VOCAB, (2, 64), generator=g).cuda() for _ in range(n)]


def lm_loss(model, ids):
    return model(input_ids=ids, labels=ids).loss


def _trainer(model, **kw):
    from usaf_b200.trainer import SparseTrainer
    args = dict(steps=20, lr_peak=1e-3, accum=2, frac=0.01, reselect_every=3)
    args.update(kw)
    tr = SparseTrainer(model, **args)
    tr.init_selection(tr.importance(_batches(1, 99)[0], lm_loss))
    return tr


def test_steps_reselect_and_skip(model):
    tr = _trainer(model)
    counts = {n: a.numel() for n, a in tr.active.items()}
    assert len(counts) == 2 * LAYERS and all(c > 0 for c in counts.values())
    m0 = {n: m.data.clone() for n, m in tr.masters.items()}
    r0 = {n: p.data.clone() for n, p in tr.router_params.items()}
    for step in (1, 2):
        out = tr.train_step(_batches(2, step), lm_loss)
        assert out["finite"] and out["step"] == step and torch.isfinite(torch.tensor(out["loss"]))
    assert tr.opt.state_dict()["step"] == 2
    assert any(not torch.equal(m0[n], tr.masters[n].data) for n in m0)
    assert any(not torch.equal(r0[n], p.data) for n, p in tr.router_params.items())
    # step 3: RigL reselection first (fresh optimizer), then the step
    old_active = {n: a.clone() for n, a in tr.active.items()}
    out = tr.train_step(_batches(2, 3), lm_loss)
    assert out["finite"]
    assert tr.opt.state_dict()["step"] == 1
    assert {n: a.numel() for n, a in tr.active.items()} == counts
    assert any(set(old_active[n].tolist()) != set(tr.active[n].tolist()) for n in counts)
    # a non-finite loss: skipped, nothing moves, the scale halves
    scale = tr.scaler.scale
    m1 = {n: m.data.clone() for n, m in tr.masters.items()}
    r1 = {n: p.data.clone() for n, p in tr.router_params.items()}
    st1 = tr.opt.state_dict()
    out = tr.train_step(_batches(2, 4), lambda mdl, ids: lm_loss(mdl, ids) * float("inf"))
    assert not out["finite"] and tr.scaler.scale == scale / 2 and tr.scaler.n_skipped == 1
    for n in m1:
        assert torch.equal(m1[n], tr.masters[n].data), n
    for n, p in tr.router_params.items():
        assert torch.equal(r1[n], p.data), n
    st2 = tr.opt.state_dict()
    assert st2["step"] == st1["step"]
    for n in st1["m"]:
        assert torch.equal(st1["m"][n], st2["m"][n])
    # the next good step proceeds at the halved scale
    out = tr.train_step(_batches(2, 5), lm_loss)
    assert out["finite"] and out["scale"] == scale / 2


def test_checkpoint_round_trip(model, tmp_path):
    from usaf_b200.trainer import SparseTrainer
    tr = _trainer(model, reselect_every=100)
    for step in (1, 2):
        tr.train_step(_batches(2, 10 + step), lm_loss)
    path = tr.save_checkpoint(str(tmp_path / "ck.pt"))
    tr2 = SparseTrainer(model, steps=20, lr_peak=1e-3, accum=2, frac=0.01, reselect_every=100)
    tr2.load_checkpoint(path)
    assert tr2.step_num == 2 and tr2.scaler.scale == tr.scaler.scale
    for n in tr.active:
        assert torch.equal(tr.active[n], tr2.active[n]), n
        assert torch.equal(tr.masters[n].data, tr2.masters[n].data), n
    s1, s2 = tr.opt.state_dict(), tr2.opt.state_dict()
    assert s1["step"] == s2["step"]
    for n in s1["m"]:
        assert torch.equal(s1["m"][n], s2["m"][n]) and torch.equal(s1["v"][n], s2["v"][n])


def test_importance_scorer_int4_experts(model):
    """ImportanceScorer (usaf/importance.py) on the patched model: the int4
    expert tensors are scored under the reference's parameter names, scores
    add over batches (two batches = the sum of each alone, bit for bit), and
    the selectors pick from them on the device."""
    from usaf_b200.importance import ImportanceScorer
    from usaf_b200.selector import TopKSelector
    dev = torch.device("cuda:0")
    bs = [{"input_ids": ids, "labels": ids} for ids in _batches(2, 77)]
    gates = {n: p for n, p in model.named_parameters() if n.endswith("mlp.gate.weight")}
    sc = ImportanceScorer(model, dev, torch.bfloat16, skip_patterns=("embed_tokens", "lm_head", "self_attn",
                                                                      "norm")).compute_scores(bs)
    one = [ImportanceScorer(model, dev, torch.bfloat16,
                            skip_patterns=("embed_tokens", "lm_head", "self_attn", "norm")).compute_scores([b])
           for b in bs]
    names = [f"model.layers.{i}.mlp.experts.{w}" for i in range(LAYERS) for w in ("gate_up_proj", "down_proj")]
    for n in names:
        shape = (E, 2 * I, H) if n.endswith("gate_up_proj") else (E, H, I)
        assert sc[n].is_cuda and tuple(sc[n].shape) == shape, n
        assert sc[n].abs().sum() > 0, n
        assert torch.equal(sc[n], one[0][n] + one[1][n]), n
    for n in gates:
        assert torch.allclose(sc[n], one[0][n] + one[1][n], rtol=1e-6, atol=0), n
    assert all(not p.requires_grad for p in model.parameters())
    for p in gates.values():     # the other tests train the gates
        p.requires_grad_(True)
    k = 1000
    masks = TopKSelector(k).select({n: sc[n] for n in names})
    assert sum(int(m.sum()) for m in masks.values()) >= k
