"""SparseTrainer against the oracle restatement of train.py's loop
(oracle/trainer.py), step by step, on a two-layer fp32 Qwen3-MoE causal LM
with int4 experts: LR warm-up + cosine, loss scaling with the division by
loss_scale * accum, accumulation over two micro-batches, SparseAdam over the
expert masters with the overlay write-back read by the next forward, and
train.py's SGD-momentum router.

Tolerances (relative Frobenius error; fp32 throughout, the attention and
norm layers run on cuBLAS / CPU BLAS in different orders): the logged loss
<= 1e-5; each step's master update (Adam moves a coordinate by ~lr * sign of
its gradient, so the update is compared rather than the masters) <= 1e-3;
the router weights' change since the start <= 1e-3 (the router gradient
of a layer sums over tokens after the fp32 attention of the layers above,
computed in other orders on the two sides: ~1e-4 apart).
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

E, K, H, I, LAYERS, VOCAB = 8, 2, 256, 128, 2, 256


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import usaf_b200  # noqa: F401
    return torch.device("cuda:0")


def _models(dev):
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeForCausalLM
    from oracle import quant as oquant
    from usaf_b200 import qwen3moe
    from usaf_b200.engine import Projection
    qwen3moe.patch_qwen3moe_for_b200()
    cfg = Qwen3MoeConfig(vocab_size=VOCAB, hidden_size=H, intermediate_size=512, num_hidden_layers=LAYERS,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                         moe_intermediate_size=I, num_experts=E, num_experts_per_tok=K,
                         norm_topk_prob=True, max_position_embeddings=128, attention_dropout=0.0)
    torch.manual_seed(0)
    cpu = Qwen3MoeForCausalLM(cfg).float().eval()
    gpu = Qwen3MoeForCausalLM(cfg).float().eval()
    gpu.load_state_dict(cpu.state_dict())
    gpu = gpu.to(dev)
    for m in (cpu, gpu):
        for p in m.parameters():
            p.requires_grad_(False)
    g = torch.Generator().manual_seed(3)
    int4, active = {}, {}
    for i in range(LAYERS):
        pre = f"model.layers.{i}.mlp.experts"
        projs = []
        for which, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
            w = (torch.randn(*shape, generator=g) * 0.02).numpy()
            q, s, z, _ = oquant.quantize_4bit(w, 128)
            int4[f"{pre}.{which}"] = oquant.dequantize_4bit(q, s, z, shape, 128)
            projs.append(Projection(torch.from_numpy(q).to(dev), torch.from_numpy(s).to(dev),
                                    torch.from_numpy(z).to(dev), shape, 128, torch.float32))
            numel = int(np.prod(shape))
            active[f"{pre}.{which}"] = torch.randperm(numel, generator=g)[: numel // 100]
        qwen3moe.attach_int4_experts(gpu.get_submodule(pre), *projs)
        gpu.get_submodule(f"model.layers.{i}.mlp").gate.weight.requires_grad_(True)
    return cpu, gpu, int4, active


def lm_loss(model, ids):
    return model(input_ids=ids, labels=ids).loss


def test_trainer_trajectory_vs_oracle(dev):
    from oracle.trainer import OracleTrainer
    from usaf_b200.trainer import SparseTrainer
    steps_total, lr, wd, accum, n_steps = 40, 1e-3, 0.005, 2, 3
    cpu, gpu, int4, active = _models(dev)
    ref = OracleTrainer(cpu, int4, active, steps_total, lr, wd, accum)
    tr = SparseTrainer(gpu, steps=steps_total, lr_peak=lr, weight_decay=wd, accum=accum, frac=0.01,
                       reselect_every=1000)
    tr.init_selection({n: a.to(dev) for n, a in active.items()})
    w0 = [cpu.get_submodule(f"model.layers.{i}.mlp").gate.weight.detach().clone() for i in range(LAYERS)]
    gen = torch.Generator().manual_seed(11)
    prev_ref = {n: m.clone() for n, m in ref.masters.items()}
    prev_dev = {n: tr.masters[n].data.cpu().clone() for n in tr.masters}
    for s in range(n_steps):
        mbs = [torch.randint(0, VOCAB, (2, 32), generator=gen) for _ in range(accum)]
        r = ref.train_step(mbs)
        d = tr.train_step([m.to(dev) for m in mbs], lm_loss)
        assert d["finite"] and r["finite"]
        assert d["lr"] == pytest.approx(r["lr"], rel=1e-12) and d["scale"] == r["scale"]
        assert abs(d["loss"] - r["loss"]) <= 1e-5 * abs(r["loss"]), (s, d["loss"], r["loss"])
        for n in active:
            # the trainer keeps its compact vectors in CSR order: align by coordinate
            a_dev = tr.active[n].cpu()
            o_dev, o_ref = a_dev.argsort(), ref.active[n].argsort()
            assert torch.equal(a_dev[o_dev], ref.active[n][o_ref])
            m_dev = tr.masters[n].data.cpu()
            upd_dev = (m_dev - prev_dev[n])[o_dev]
            upd_ref = (ref.masters[n] - prev_ref[n])[o_ref]
            assert upd_ref.abs().max() > 0
            r_upd = rel(upd_dev, upd_ref)
            assert r_upd <= 1e-3, f"step {s} {n}: master update rel {r_upd:.2e}"
            prev_dev[n], prev_ref[n] = m_dev.clone(), ref.masters[n].clone()
        for i in range(LAYERS):
            wg = gpu.get_submodule(f"model.layers.{i}.mlp").gate.weight.detach().cpu()
            wc = cpu.get_submodule(f"model.layers.{i}.mlp").gate.weight.detach()
            r_w = rel(wg - w0[i], wc - w0[i])
            assert r_w <= 1e-3, f"step {s} layer {i}: router update rel {r_w:.2e}"
