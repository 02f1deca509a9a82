"""``usaf train`` on the B200 path (drop-in for usaf/train.py:38-171).

The parser, ``TrainConfig`` and ``parse_args`` keep the reference's flags,
defaults and field names (usaf/train.py:38-171), so a command line written
for the reference parses to the same configuration here.  ``main`` runs the
sparse training of a Qwen3-MoE model on the device kernels:

* ``--model``: a local Hugging Face model directory (``config.json``, and the
  non-expert weights in ``*.safetensors`` when present; without weight files
  the non-expert layers keep their seeded random init and a notice says so).
  There is no network access and no model download.
* ``--quant-path`` (default ``<model name>-q4/experts_q4.pt``, as the
  reference): the int4 expert store in the usaf.quantization layout, one
  entry per ``model.layers.{i}.mlp.experts.{gate_up_proj,down_proj}``; the
  experts live in HBM as :class:`usaf_b200.engine.Projection`.
* ``--dataset``: the reference's JSONL of tokenized samples
  (``input_ids`` of length ``--seq-len``, ``labels`` optional), shuffled with
  seed 42 and split into train / eval / held-out as usaf/train.py:173-194.
* training: :class:`usaf_b200.trainer.SparseTrainer` -- importance selection
  of ``--frac`` on the first micro-batch, LR warm-up + cosine, loss scaling,
  ``--accum`` micro-batches of ``--microbatch`` samples, RigL every
  ``--reselect-every`` steps, SGD-momentum router; layers from
  ``--train-from`` (0: all) are trained.
* outputs: a JSONL log per step in ``--log-dir``, ``usaf-sparse-v1``
  checkpoints every ``--save-every`` steps and at the end in
  ``--checkpoint-dir``, ``--resume`` from such a file, ``--export`` of the
  merged int4 experts (usaf/checkpoint.py:58-92).
* ``--eval-only``: perplexity of the eval and held-out samples.

Flags of the reference's host-memory machinery have nothing to act on here
and are accepted and recorded only: ``--no-frozen-cache``,
``--frozen-cache-n`` (frozen-layer activation cache), ``--no-resident``
(the experts are always resident in HBM), ``--no-amp`` (bf16 throughout),
``--no-multi-gpu`` (several GPUs run expert-parallel under
``torch.distributed.run``).  ``--no-cuda`` raises: there is no CPU path.

    python -m usaf_b200.train --model ./tiny-qwen3moe --dataset data.jsonl --steps 20
"""
from __future__ import annotations

import argparse
import json
import math
import os
import random
import sys
import time
from dataclasses import asdict, dataclass
from typing import List, Optional, Tuple

import torch


def build_parser() -> argparse.ArgumentParser:
    """usaf/train.py:38-94: the same flags and defaults."""
    p = argparse.ArgumentParser(description="USAF: Ultra Sparse Adaptive Fine-Tuning (B200)")
    p.add_argument("--model", type=str, required=True,
                   help="local Hugging Face model directory (config.json [+ *.safetensors])")
    p.add_argument("--dataset", type=str, required=True, help="Path to JSONL dataset file")
    p.add_argument("--quant-path", type=str, default="",
                   help="Path to q4 experts file. Auto-detected if empty.")
    p.add_argument("--steps", type=int, default=180)
    p.add_argument("--epochs", type=float, default=0,
                   help="If >0, overrides --steps based on dataset size")
    p.add_argument("--seq-len", type=int, default=512)
    p.add_argument("--microbatch", type=int, default=2)
    p.add_argument("--accum", type=int, default=1)
    p.add_argument("--frac", type=float, default=0.005)
    p.add_argument("--lr", type=float, default=2e-4)
    p.add_argument("--wd", type=float, default=0.005)
    p.add_argument("--train-from", type=int, default=0, help="First trainable layer (0=auto)")
    p.add_argument("--reselect-every", type=int, default=50)
    p.add_argument("--no-frozen-cache", action="store_true")
    p.add_argument("--no-resident", action="store_true")
    p.add_argument("--frozen-cache-n", type=int, default=0)
    p.add_argument("--eval-every", type=int, default=15)
    p.add_argument("--cuda", action="store_true", default=None)
    p.add_argument("--no-cuda", action="store_true", default=None)
    p.add_argument("--no-amp", action="store_true")
    p.add_argument("--no-multi-gpu", action="store_true")
    p.add_argument("--tag", type=str, default="")
    p.add_argument("--checkpoint-dir", type=str, default="checkpoints")
    p.add_argument("--log-dir", type=str, default="logs")
    p.add_argument("--resume", type=str, default="",
                   help="Path to sparse checkpoint to resume from")
    p.add_argument("--save-every", type=int, default=50,
                   help="Save checkpoint every N steps (0=no mid-training saves)")
    p.add_argument("--export", type=str, default="",
                   help="Export merged weights path (e.g. experts_finetuned_q4.pt)")
    p.add_argument("--eval-only", action="store_true",
                   help="Skip training, only evaluate model/checkpoint")
    p.add_argument("--eval-datasets", type=str, default="synthetic-cpp",
                   help="Comma-separated list of eval datasets")
    p.add_argument("--eval-samples", type=int, default=64, help="Max samples per eval dataset")
    p.add_argument("--eval-report", type=str, default="", help="Path to save eval report JSON")
    return p


@dataclass
class TrainConfig:
    """usaf/train.py:97-128: the same fields and defaults."""
    model_path: str
    dataset_path: str
    quant_path: str = ""
    steps: int = 180
    epochs: float = 0
    seq_len: int = 512
    microbatch: int = 2
    accum: int = 1
    frac: float = 0.005
    lr_peak: float = 2e-4
    weight_decay: float = 0.005
    train_from: int = 0
    reselect_every: int = 50
    use_frozen_cache: bool = True
    frozen_cache_n: int = 0
    use_resident: bool = True
    eval_every: int = 15
    use_cuda: Optional[bool] = None
    use_amp: bool = True
    use_multi_gpu: bool = True
    tag: str = ""
    checkpoint_dir: str = "checkpoints"
    log_dir: str = "logs"
    resume_path: str = ""
    save_every: int = 50
    export_path: str = ""
    eval_only: bool = False
    eval_datasets: str = "synthetic-cpp"
    eval_samples: int = 64
    eval_report: str = ""


def parse_args(args=None) -> TrainConfig:
    """usaf/train.py:131-171: ``--cuda`` / ``--no-cuda`` resolve to
    ``use_cuda`` (default: whether a CUDA device is visible)."""
    ns = build_parser().parse_args(args)
    use_cuda = ns.cuda
    if use_cuda is None and ns.no_cuda:
        use_cuda = False
    if use_cuda is None:
        use_cuda = torch.cuda.is_available()
    return TrainConfig(
        model_path=ns.model, dataset_path=ns.dataset, quant_path=ns.quant_path, steps=ns.steps,
        epochs=ns.epochs, seq_len=ns.seq_len, microbatch=ns.microbatch, accum=ns.accum,
        frac=ns.frac, lr_peak=ns.lr, weight_decay=ns.wd, train_from=ns.train_from,
        reselect_every=ns.reselect_every, use_frozen_cache=not ns.no_frozen_cache,
        frozen_cache_n=ns.frozen_cache_n, use_resident=not ns.no_resident,
        eval_every=ns.eval_every, use_cuda=use_cuda, use_amp=not ns.no_amp,
        use_multi_gpu=not ns.no_multi_gpu, tag=ns.tag, checkpoint_dir=ns.checkpoint_dir,
        log_dir=ns.log_dir, resume_path=ns.resume, save_every=ns.save_every,
        export_path=ns.export, eval_only=ns.eval_only, eval_datasets=ns.eval_datasets,
        eval_samples=ns.eval_samples, eval_report=ns.eval_report)


def load_dataset(path: str, seq_len: int) -> Tuple[list, list, list]:
    """usaf/train.py:173-194: JSONL samples whose ``input_ids`` have exactly
    ``seq_len`` tokens (other lines are skipped), shuffled with seed 42; the
    last 20 samples are the eval (10) and held-out (10) sets."""
    samples = []
    if os.path.exists(path):
        with open(path) as f:
            for line in f:
                line = line.strip()
                if not line:
                    continue
                try:
                    s = json.loads(line)
                except json.JSONDecodeError:
                    continue
                if "input_ids" in s and len(s["input_ids"]) == seq_len:
                    samples.append(s)
    rng = random.Random(42)
    rng.shuffle(samples)
    n_train = max(1, len(samples) - 20)
    return samples[:n_train], samples[n_train:n_train + 10], samples[n_train + 10:n_train + 20]


def _batch(samples, device) -> dict:
    ids = torch.tensor([s["input_ids"] for s in samples], dtype=torch.long, device=device)
    labels = torch.tensor([s.get("labels", s["input_ids"]) for s in samples], dtype=torch.long,
                          device=device)
    return {"input_ids": ids, "labels": labels}


def lm_loss(model, batch) -> torch.Tensor:
    return model(input_ids=batch["input_ids"], labels=batch["labels"]).loss


def load_model(config: TrainConfig, device):
    """Qwen3-MoE model on the device with int4 experts attached from the q4
    store; returns (model, q4 path, the expert modules to train: layers from
    --train-from on)."""
    from transformers import AutoConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeForCausalLM
    from . import qwen3moe
    cfg = AutoConfig.from_pretrained(config.model_path)
    if getattr(cfg, "model_type", "") != "qwen3_moe":
        raise ValueError(f"{config.model_path}: model_type {getattr(cfg, 'model_type', '?')!r}; "
                         "the B200 path trains Qwen3-MoE models")
    qwen3moe.patch_qwen3moe_for_b200()
    torch.manual_seed(0)
    with torch.device(device), qwen3moe.without_dense_experts():
        model = Qwen3MoeForCausalLM(cfg).to(torch.bfloat16)
    weights = sorted(f for f in os.listdir(config.model_path) if f.endswith(".safetensors"))
    if weights:
        from safetensors.torch import load_file
        sd = {}
        for f in weights:
            sd.update({k: v for k, v in load_file(os.path.join(config.model_path, f)).items()
                       if ".mlp.experts." not in k})
        missing = model.load_state_dict(sd, strict=False)
        print(f"  weights: {len(sd)} tensors from {len(weights)} file(s); "
              f"{len(missing.missing_keys)} left at init")
    else:
        print("  weights: none found, the non-expert layers keep their seeded random init")
    for p in model.parameters():
        p.requires_grad_(False)
    quant = config.quant_path or f"{config.model_path.rstrip('/').split('/')[-1]}-q4/experts_q4.pt"
    q_dict = torch.load(quant, map_location="cpu", weights_only=True)
    n_layers = cfg.num_hidden_layers
    first = config.train_from if config.train_from > 0 else 0
    names: List[str] = []
    for i in range(n_layers):
        pre = f"model.layers.{i}.mlp.experts"
        gu_e, dn_e = q_dict[f"{pre}.gate_up_proj"], q_dict[f"{pre}.down_proj"]
        shape_of = (lambda e: tuple(e["shape"]) if isinstance(e, dict) else tuple(e[3]))
        gu = qwen3moe.int4_projection(gu_e, shape_of(gu_e), device=device)
        dn = qwen3moe.int4_projection(dn_e, shape_of(dn_e), device=device)
        qwen3moe.attach_int4_experts(model.get_submodule(pre), gu, dn)
        if i >= first:
            names.append(pre)
            model.get_submodule(f"model.layers.{i}.mlp").gate.weight.requires_grad_(True)
    return model, quant, names


@torch.no_grad()
def eval_ppl(model, samples, device, n: int) -> Tuple[float, float]:
    tot = 0.0
    k = 0
    for s in samples[:n]:
        tot += float(lm_loss(model, _batch([s], device)))
        k += 1
    loss = tot / max(k, 1)
    return loss, math.exp(min(loss, 50.0))


def main(args=None):
    config = parse_args(args)
    if not config.use_cuda:
        raise SystemExit("usaf_b200 trains on CUDA (B200) only; there is no CPU path")
    from . import checkpoint as ckpt
    from .trainer import SparseTrainer
    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    print("=" * 60)
    print("USAF (B200) - Ultra Sparse Adaptive Fine-Tuning")
    print("=" * 60)
    train, evals, held = load_dataset(config.dataset_path, config.seq_len)
    if not train or "input_ids" not in train[0]:
        raise SystemExit(f"{config.dataset_path}: no samples of {config.seq_len} tokens")
    if config.epochs > 0:
        eff = config.microbatch * config.accum
        config.steps = max(1, int(config.epochs * len(train) * config.seq_len / (eff * config.seq_len)))
    print(f"Model: {config.model_path}")
    model, quant, names = load_model(config, device)
    model.train()
    if config.eval_only:
        el, ep = eval_ppl(model, evals, device, config.eval_samples)
        hl, hp = eval_ppl(model, held, device, config.eval_samples)
        rep = {"eval_loss": el, "eval_ppl": ep, "heldout_loss": hl, "heldout_ppl": hp}
        print(json.dumps(rep))
        if config.eval_report:
            with open(config.eval_report, "w") as f:
                json.dump(rep, f, indent=2)
        return model
    tr = SparseTrainer(model, steps=config.steps, lr_peak=config.lr_peak,
                       weight_decay=config.weight_decay, accum=config.accum, frac=config.frac,
                       reselect_every=config.reselect_every, expert_names=names)
    os.makedirs(config.log_dir, exist_ok=True)
    os.makedirs(config.checkpoint_dir, exist_ok=True)
    tag = config.tag or time.strftime("%Y%m%d_%H%M%S")
    log_path = os.path.join(config.log_dir, f"train_{tag}.jsonl")
    ck_path = os.path.join(config.checkpoint_dir, f"usaf_sparse_{tag}.pt")
    si = 0

    def next_micro():
        nonlocal si
        mb = [train[(si + j) % len(train)] for j in range(config.microbatch)]
        si += config.microbatch
        return _batch(mb, device)

    if config.resume_path and os.path.exists(config.resume_path):
        tr.load_checkpoint(config.resume_path)
        si = tr.step_num * config.accum * config.microbatch
        print(f"Resumed at step {tr.step_num}")
    else:
        tr.init_selection(tr.importance(next_micro(), lm_loss))
    n_act = sum(a.numel() for a in tr.active.values())
    print(f"Active: {n_act:,} coordinates in {len(tr.active)} expert tensors; "
          f"steps {config.steps}, batch {config.microbatch}x{config.accum}")
    with open(log_path, "a") as log:
        log.write(json.dumps({"config": asdict(config)}) + "\n")
        while tr.step_num < config.steps:
            t0 = time.time()
            out = tr.train_step([next_micro() for _ in range(config.accum)], lm_loss)
            dt = time.time() - t0
            out["sec"] = round(dt, 3)
            out["tok_s"] = round(config.accum * config.microbatch * config.seq_len / max(dt, 1e-9), 1)
            if config.eval_every and out["step"] % config.eval_every == 0 and evals:
                out["eval_loss"], out["eval_ppl"] = eval_ppl(model, evals, device, config.eval_samples)
            log.write(json.dumps(out) + "\n")
            log.flush()
            print(f"  step {out['step']:4d}/{config.steps} | loss {out['loss']:.4f} | lr {out['lr']:.2e} | "
                  f"{out['tok_s']:.0f} tok/s", flush=True)
            if config.save_every and out["step"] % config.save_every == 0:
                tr.save_checkpoint(ck_path)
    tr.save_checkpoint(ck_path)
    print(f"Checkpoint: {ck_path}")
    if config.export_path:
        ckpt.export_merged_weights(quant, {n_: m.data for n_, m in tr.masters.items()}, tr.active,
                                   config.export_path, device=device)
        print(f"Exported merged experts: {config.export_path}")
    return model


if __name__ == "__main__":
    main(sys.argv[1:])
