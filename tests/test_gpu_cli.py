"""`python -m usaf_b200.train` end to end on a tiny Qwen3-MoE model directory
(config.json, no weight files) with an int4 expert store and a JSONL
dataset: training steps with importance selection and a RigL step, the
per-step log, usaf-sparse-v1 checkpoints, resume, the merged int4 export
and the eval-only report."""
import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu

E, K, H, I, LAYERS, VOCAB, SEQ = 8, 2, 256, 128, 2, 128, 32


@pytest.fixture(scope="module")
def setup(tmp_path_factory):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from usaf_b200.quantization import quantize_4bit
    d = tmp_path_factory.mktemp("cli")
    model_dir = d / "tiny-qwen3moe"
    Qwen3MoeConfig(vocab_size=VOCAB, hidden_size=H, intermediate_size=512, num_hidden_layers=LAYERS,
                   num_attention_heads=4, num_key_value_heads=2, head_dim=64, moe_intermediate_size=I,
                   num_experts=E, num_experts_per_tok=K, norm_topk_prob=True,
                   max_position_embeddings=128).save_pretrained(str(model_dir))
    g = torch.Generator(device="cuda").manual_seed(0)
    q4 = {}
    for i in range(LAYERS):
        for which, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
            w = torch.randn(*shape, device="cuda", generator=g) * 0.02
            q, s, z, sh = quantize_4bit(w, 128)
            q4[f"model.layers.{i}.mlp.experts.{which}"] = {"q": q.cpu(), "s": s.cpu(), "z": z.cpu(),
                                                          "shape": tuple(sh), "group_size": 128}
    quant = d / "experts_q4.pt"
    torch.save(q4, str(quant))
    rng = torch.Generator().manual_seed(1)
    data = d / "data.jsonl"
    with open(data, "w") as f:
        for _ in range(48):
            f.write(json.dumps({"input_ids": torch.randint(0, VOCAB, (SEQ,), generator=rng).tolist()}) + "\n")
    return d, model_dir, quant, data


def _args(setup, *extra):
    d, model_dir, quant, data = setup
    return ["--model", str(model_dir), "--dataset", str(data), "--quant-path", str(quant),
            "--seq-len", str(SEQ), "--microbatch", "2", "--accum", "2", "--frac", "0.01",
            "--lr", "1e-3", "--reselect-every", "3", "--eval-every", "2", "--eval-samples", "4",
            "--checkpoint-dir", str(d / "ck"), "--log-dir", str(d / "logs"), *extra]


def test_train_resume_export_eval(setup):
    from usaf_b200 import checkpoint, train
    d = setup[0]
    train.main(_args(setup, "--steps", "4", "--save-every", "2", "--tag", "a",
                     "--export", str(d / "merged_q4.pt")))
    rows = [json.loads(line) for line in open(d / "logs" / "train_a.jsonl")]
    steps = [r for r in rows if "step" in r]
    assert [r["step"] for r in steps] == [1, 2, 3, 4]
    assert all(r["finite"] and r["loss"] == r["loss"] for r in steps)
    assert "eval_ppl" in steps[1]
    ck = d / "ck" / "usaf_sparse_a.pt"
    meta = checkpoint.get_checkpoint_metadata(str(ck))
    assert meta["format"] == "usaf-sparse-v1" and meta["step"] == 4 and meta["n_active"] > 0
    merged = torch.load(str(d / "merged_q4.pt"), weights_only=True)
    assert set(merged) == set(torch.load(str(setup[2]), weights_only=True))
    # resume: two more steps from the step-4 checkpoint
    train.main(_args(setup, "--steps", "6", "--tag", "a", "--resume", str(ck)))
    assert checkpoint.get_checkpoint_metadata(str(ck))["step"] == 6
    # eval only
    rep = d / "rep.json"
    train.main(_args(setup, "--eval-only", "--eval-report", str(rep)))
    r = json.load(open(rep))
    assert r["eval_ppl"] > 1 and r["heldout_ppl"] > 1
