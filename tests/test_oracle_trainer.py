"""The oracle restatement of train.py's loop (oracle/trainer.py) on the CPU:
it trains (losses finite, masters and routers move, the LR follows the
warm-up), the overlay write-back reaches the next forward (a master moved by
hand changes the next loss), and a non-finite step is skipped with the loss
scale halved (train.py:661-677)."""
import numpy as np
import pytest
import torch

E, K, H, I, VOCAB = 4, 2, 128, 128, 64


def _tiny():
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeForCausalLM
    from oracle import quant as oquant
    cfg = Qwen3MoeConfig(vocab_size=VOCAB, hidden_size=H, intermediate_size=256, num_hidden_layers=1,
                         num_attention_heads=2, num_key_value_heads=1, head_dim=64,
                         moe_intermediate_size=I, num_experts=E, num_experts_per_tok=K,
                         norm_topk_prob=True, max_position_embeddings=64, attention_dropout=0.0)
    torch.manual_seed(0)
    m = Qwen3MoeForCausalLM(cfg).float().eval()
    for p in m.parameters():
        p.requires_grad_(False)
    g = torch.Generator().manual_seed(1)
    int4, active = {}, {}
    pre = "model.layers.0.mlp.experts"
    for which, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = (torch.randn(*shape, generator=g) * 0.02).numpy()
        q, s, z, _ = oquant.quantize_4bit(w, 128)
        int4[f"{pre}.{which}"] = oquant.dequantize_4bit(q, s, z, shape, 128)
        active[f"{pre}.{which}"] = torch.randperm(int(np.prod(shape)), generator=g)[:500]
    return m, int4, active


def test_oracle_trainer_steps_and_skip():
    from oracle.trainer import OracleTrainer, lr_at
    m, int4, active = _tiny()
    tr = OracleTrainer(m, int4, active, steps=40, lr_peak=1e-3, weight_decay=0.005, accum=2)
    gate = m.model.layers[0].mlp.gate.weight
    g0 = gate.detach().clone()
    m0 = {n: v.clone() for n, v in tr.masters.items()}
    gen = torch.Generator().manual_seed(2)
    batch = lambda: [torch.randint(0, VOCAB, (2, 16), generator=gen) for _ in range(2)]  # noqa: E731
    for step in (1, 2):
        out = tr.train_step(batch())
        assert out["finite"] and np.isfinite(out["loss"])
        assert out["lr"] == pytest.approx(lr_at(step, 40, 1e-3))
    assert not torch.equal(gate.detach(), g0)
    assert all(not torch.equal(m0[n], tr.masters[n]) for n in m0)
    # write-back: moving one master moves the next forward's loss
    ids = torch.randint(0, VOCAB, (2, 16), generator=gen)
    tr._sync_resident()
    base = float(m(input_ids=ids, labels=ids).loss)
    n = next(iter(tr.masters))
    tr.masters[n].add_(0.5)
    tr._sync_resident()
    assert float(m(input_ids=ids, labels=ids).loss) != base
    tr.masters[n].sub_(0.5)
    # a non-finite step: no update, the scale halves
    scale = tr.scale
    snap = {k: v.clone() for k, v in tr.masters.items()}
    g1 = gate.detach().clone()
    nan_ids = [torch.randint(0, VOCAB, (2, 16), generator=gen) for _ in range(2)]
    orig = tr.model.forward

    def bad_forward(*a, **kw):
        o = orig(*a, **kw)
        o.loss = o.loss * float("inf")
        return o
    tr.model.forward = bad_forward
    try:
        out = tr.train_step(nan_ids)
    finally:
        tr.model.forward = orig
    assert not out["finite"] and tr.scale == scale / 2
    assert all(torch.equal(snap[k], tr.masters[k]) for k in snap)
    assert torch.equal(gate.detach(), g1)
