"""Generate golden fixtures by running the REFERENCE implementation.

Run in the build container, where the reference checkout is importable:

    python tests/golden/make_golden.py --reference /path/to/usaf

It imports the reference's own modules (``usaf.qwen3moe_dml``,
``usaf.quantization``, ``usaf.moe_loader``, ``usaf.sparse_optim``) and the
batched-dispatch forward of ``benchmarks/kaggle_t4_bench.py`` (extracted from
the script with ``ast`` and instrumented to expose its dispatch tensors), runs
them on the seeded inputs of ``oracle.inputs`` and writes their outputs to
``tests/golden/*.pt``.  Only outputs and input hashes are stored; tests
regenerate the inputs from the seed.  Nothing here runs on the GPU box.
"""
from __future__ import annotations

import argparse
import ast
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle.inputs import make_block_inputs, C1  # noqa: E402


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def load_batched_dispatch(ref_root):
    """Extract ``batched_sparse_experts_forward`` from the reference benchmark
    script and make every ``return`` first publish its local tensors."""
    path = os.path.join(ref_root, "benchmarks", "kaggle_t4_bench.py")
    tree = ast.parse(open(path).read())
    fn = next(n for n in ast.walk(tree)
              if isinstance(n, ast.FunctionDef) and n.name == "batched_sparse_experts_forward")

    class Tap(ast.NodeTransformer):
        def visit_Return(self, node):
            tap = ast.parse("__golden__.update({k: v for k, v in locals().items() "
                            "if isinstance(v, torch.Tensor)})").body[0]
            return [tap, node]

    fn = Tap().visit(fn)
    mod = ast.Module(body=[fn], type_ignores=[])
    ast.fix_missing_locations(mod)
    ns = {"torch": torch, "__golden__": {}}
    exec(compile(mod, path, "exec"), ns)
    return ns["batched_sparse_experts_forward"], ns["__golden__"]


def run_case(ref_root, cfg, frac=0.005, lr=1e-4):
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from usaf.qwen3moe_dml import patch_qwen3moe_for_dml
    from usaf.quantization import quantize_4bit as ref_quant, dequantize_4bit as ref_deq
    from usaf.moe_loader import SparseGradStore, TopKImportanceStore
    from usaf.sparse_optim import SparseAdam

    mq = patch_qwen3moe_for_dml()
    inp = make_block_inputs(**cfg)
    H, E, k, I, T, dt = inp["H"], inp["E"], inp["k"], inp["I"], inp["T"], inp["dtype"]

    # regenerate the fp32 expert weights and quantize them with the REFERENCE quantizer
    torch.manual_seed(cfg["seed"])
    if cfg.get("order") == "c1":
        _ = torch.randn(E, H)
        w_gu = torch.randn(E, 2 * I, H) * 0.02
        w_dn = torch.randn(E, H, I) * 0.02
    else:
        _ = torch.randn(T, H)
        _ = torch.randn(E, H)
        w_gu = torch.randn(E, 2 * I, H) * 0.02
        w_dn = torch.randn(E, H, I) * 0.02
    g = {"meta": {"cfg": {k_: (str(v) if isinstance(v, torch.dtype) else v) for k_, v in cfg.items()}}}
    deq = {}
    for name, w in (("gate_up_proj", w_gu), ("down_proj", w_dn)):
        q, s, z, shape = ref_quant(w, 128)
        g[f"{name}.qsz_sha"] = sha(q.numpy(), s.numpy(), z.numpy())
        deq[name] = ref_deq(q, s, z, shape, 128)
        g[f"{name}.deq_sha"] = sha(deq[name].numpy())

    mcfg = Qwen3MoeConfig(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                          moe_intermediate_size=I, norm_topk_prob=True)
    blk = mq.Qwen3MoeSparseMoeBlock(mcfg).to(dt)
    prefix = "layer.mlp.experts"
    shapes = {f"{prefix}.gate_up_proj": (E, 2 * I, H), f"{prefix}.down_proj": (E, H, I)}
    with torch.no_grad():
        blk.gate.weight.copy_(inp["w_r"])
        # the dequantized int4 weights are fp16; the block computes in the
        # activation dtype, so they are cast fp16 -> activation dtype
        blk.experts.gate_up_proj.copy_(deq["gate_up_proj"].to(dt))
        blk.experts.down_proj.copy_(deq["down_proj"].to(dt))

    seen = {}
    orig_fwd = blk.experts.forward

    def tap(hs, weights):
        seen["weights"] = weights.detach().clone()
        return orig_fwd(hs, weights)
    blk.experts.forward = tap

    x = inp["x"].reshape(1, T, H)
    dy = inp["dy"].reshape(1, T, H)

    # importance pass (train.py:397-402) with the reference store
    imp = TopKImportanceStore(shapes, frac=frac)
    blk.experts._grad_capture = (imp, prefix)
    xi = x.clone().requires_grad_(True)
    blk.zero_grad(set_to_none=True)
    y0 = blk(xi)
    y0.backward(dy)
    active = imp.select(frac)
    for n in shapes:
        g[f"cand.{n}.vals"] = torch.cat(list(imp._vals[n].values()))
        g[f"cand.{n}.idx"] = torch.cat(list(imp._idx[n].values()))
        g[f"cand.{n}.experts"] = torch.tensor(list(imp._vals[n].keys()))
        g[f"active.{n}"] = active[n].clone()

    # masters from the original dequant (train.py:451-467)
    masters = {n: torch.nn.Parameter(deq[n.rsplit(".", 1)[1]].reshape(-1)
                                     .index_select(0, active[n]).float(), requires_grad=False)
               for n in shapes}

    # training pass with the sparse store (train.py:408-412, 631-641)
    store = SparseGradStore(active, shapes)
    blk.experts._grad_capture = (store, prefix)
    xt = x.clone().requires_grad_(True)
    blk.zero_grad(set_to_none=True)
    y = blk(xt)
    y.backward(dy)
    g["weights"] = seen["weights"]
    g["y"] = y.detach().reshape(T, H).clone()
    g["dX"] = xt.grad.detach().reshape(T, H).clone()
    g["dW_r"] = blk.gate.weight.grad.detach().clone()
    for n in shapes:
        g[f"compact.{n}"] = store.compact[n].clone()

    # SparseAdam over the masters (compact mode) and the full router (gather mode)
    opt = SparseAdam(masters, active_idx=active, lr=lr, compact_params=True)
    opt.step(compact_grads={n: store.compact[n] for n in shapes})
    for n in shapes:
        g[f"master_after.{n}"] = masters[n].detach().clone()
    rname = "layer.mlp.gate.weight"
    ropt = SparseAdam({rname: blk.gate.weight}, active_idx={rname: torch.arange(E * H)}, lr=lr)
    ropt.step()
    g["w_r_after"] = blk.gate.weight.detach().clone()

    # reference batched dispatch: indices and output
    fwd, tapd = load_batched_dispatch(ref_root)

    class Shim:
        pass
    shim = Shim()
    shim.num_experts = E
    shim.gate_up_proj = blk.experts.gate_up_proj.detach()
    shim.down_proj = blk.experts.down_proj.detach()
    shim.act_fn = blk.experts.act_fn
    with torch.no_grad():
        yb = fwd(shim, inp["x"], g["weights"])
    g["y_batched"] = yb.clone()
    for key in ("tok_idx", "exp_idx", "counts", "order", "offs", "pos", "pad_tok"):
        g[f"dispatch.{key}"] = tapd[key].clone()
    return g


def run_ties(ref_root):
    """Router known answer with exact ties at the k-th place (usaf/qwen3moe_dml.py:77-79)."""
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from usaf.qwen3moe_dml import patch_qwen3moe_for_dml
    mq = patch_qwen3moe_for_dml()
    H, E, k, T = 128, 8, 2, 16
    torch.manual_seed(7)
    w_r = (torch.randn(E, H) * 0.02).to(torch.bfloat16)
    w_r[3] = w_r[1]
    w_r[5] = w_r[1]
    x = torch.randn(T, H).to(torch.bfloat16)
    mcfg = Qwen3MoeConfig(hidden_size=H, num_experts=E, num_experts_per_tok=k,
                          moe_intermediate_size=128, norm_topk_prob=True)
    blk = mq.Qwen3MoeSparseMoeBlock(mcfg).to(torch.bfloat16)
    with torch.no_grad():
        blk.gate.weight.copy_(w_r)
        blk.experts.gate_up_proj.normal_(0, 0.02)
        blk.experts.down_proj.normal_(0, 0.02)
    seen = {}
    orig = blk.experts.forward

    def tap(hs, weights):
        seen["weights"] = weights.detach().clone()
        return orig(hs, weights)
    blk.experts.forward = tap
    with torch.no_grad():
        blk(x.reshape(1, T, H))
    return {"seed": 7, "H": H, "E": E, "k": k, "T": T, "weights": seen["weights"]}


def load_rigl_merge(ref_root):
    """The per-tensor merge loop of train.py's ``do_reselect`` (train.py:552-596),
    extracted with ``ast`` and run as it is written: the ``for fname, old in
    active_idx.items():`` statement, executed in a namespace that provides the
    names it reads (``active_idx``, ``new_idx``, ``masters``, ``q_dict``,
    ``dequantize_4bit``) and collects the ones it writes (``_new_active``,
    ``_new_masters``)."""
    path = os.path.join(ref_root, "train.py")
    tree = ast.parse(open(path).read())
    fn = next(n for n in ast.walk(tree)
              if isinstance(n, ast.FunctionDef) and n.name == "do_reselect")
    loop = next(n for n in fn.body if isinstance(n, ast.For)
                and isinstance(n.target, ast.Tuple)
                and [e.id for e in n.target.elts] == ["fname", "old"])
    mod = ast.Module(body=[loop], type_ignores=[])
    ast.fix_missing_locations(mod)
    return compile(mod, path, "exec")


def run_rigl(ref_root):
    """RigL merge known answers from the reference's own loop on C1-shaped
    tensors.  Cases: (a) half of the new selection overlaps the old one;
    (b) the new selection is smaller than the old one, so fewer coordinates
    grow than were dropped; (c) no new selection (the tensor keeps its set)."""
    from usaf.quantization import quantize_4bit as ref_quant, dequantize_4bit as ref_deq
    code = load_rigl_merge(ref_root)
    inp = make_block_inputs(**C1)
    shapes = {"t.gate_up_proj": inp["gate_up_proj"]["shape"],
              "t.down_proj": inp["down_proj"]["shape"],
              "t.keep": inp["down_proj"]["shape"]}
    g = torch.Generator().manual_seed(23)
    active_idx, new_idx, masters, q_dict = {}, {}, {}, {}
    sizes = {"t.gate_up_proj": (10485, 10485), "t.down_proj": (5242, 3000), "t.keep": (5242, 0)}
    for fname, shape in shapes.items():
        numel = int(np.prod(shape))
        n_old, n_new = sizes[fname]
        perm = torch.randperm(numel, generator=g)
        old = perm[:n_old]
        # half of the new selection from the old set, half from outside it
        n_in = n_new // 2
        new = torch.cat([old[torch.randperm(n_old, generator=g)[:n_in]],
                         perm[n_old:n_old + n_new - n_in]])
        new = new[torch.randperm(new.numel(), generator=g)]
        active_idx[fname] = old
        if n_new:
            new_idx[fname] = new
        masters[fname] = torch.nn.Parameter(torch.randn(n_old, generator=g) * 0.02,
                                            requires_grad=False)
        src = "gate_up_proj" if fname.endswith("gate_up_proj") else "down_proj"
        w = torch.from_numpy(inp[src]["fp16"].astype(np.float32)) + 0.0
        q, s, z, sh = ref_quant(w, 128)
        q_dict[fname] = {"q": q, "s": s, "z": z, "shape": sh}
    ns = {"torch": torch, "active_idx": active_idx, "new_idx": new_idx, "masters": masters,
          "q_dict": q_dict, "dequantize_4bit": ref_deq, "_new_active": {}, "_new_masters": {},
          "_n_kept": 0, "_n_dropped": 0, "_n_grown": 0}
    exec(code, ns)
    out = {"names": list(shapes)}
    for fname in shapes:
        out[f"{fname}.old"] = active_idx[fname].clone()
        out[f"{fname}.new"] = new_idx[fname].clone() if fname in new_idx else None
        out[f"{fname}.masters"] = masters[fname].detach().clone()
        # the int4 entry is not stored: tests re-quantize the C1 dequant with the
        # oracle's quantizer and check it against this hash
        out[f"{fname}.qsz_sha"] = sha(q_dict[fname]["q"].numpy(), q_dict[fname]["s"].numpy(),
                                      q_dict[fname]["z"].numpy())
        out[f"{fname}.shape"] = tuple(q_dict[fname]["shape"])
        out[f"{fname}.final"] = ns["_new_active"][fname].clone()
        out[f"{fname}.final_masters"] = ns["_new_masters"][fname].detach().float().clone()
    return out


CLI_ARGS = [
    ["--model", "Qwen/Qwen3-30B-A3B", "--dataset", "data/train.jsonl"],
    ["--model", "m", "--dataset", "d.jsonl", "--steps", "360", "--epochs", "1.5", "--seq-len", "256",
     "--microbatch", "4", "--accum", "8", "--frac", "0.01", "--lr", "1e-4", "--wd", "0.01",
     "--train-from", "12", "--reselect-every", "25", "--no-frozen-cache", "--no-resident",
     "--frozen-cache-n", "3", "--eval-every", "5", "--cuda", "--no-amp", "--no-multi-gpu", "--tag", "x",
     "--checkpoint-dir", "ck", "--log-dir", "lg", "--resume", "r.pt", "--save-every", "10",
     "--export", "e.pt", "--eval-only", "--eval-datasets", "a,b", "--eval-samples", "8",
     "--eval-report", "rep.json"],
    ["--model", "m", "--dataset", "d", "--no-cuda", "--quant-path", "q.pt"],
]


def cli_dataset_lines():
    """A seeded JSONL: samples of 8 tokens, some of other lengths, a blank and
    a malformed line (the loader skips those)."""
    import json
    import random as _r
    rng = _r.Random(5)
    lines = []
    for i in range(46):
        n = 8 if i % 7 else 6
        lines.append(json.dumps({"input_ids": [rng.randrange(100) for _ in range(n)], "id": i}))
    lines.insert(10, "")
    lines.insert(20, "{not json")
    return lines


def run_cli(ref_root):
    """The reference CLI's own parse_args on CLI_ARGS (usaf/train.py:131-171)
    and its dataset loader (:173-194) on cli_dataset_lines()."""
    import dataclasses
    import tempfile
    import usaf.train as ut
    out = {"args": CLI_ARGS, "configs": [dataclasses.asdict(ut.parse_args(a)) for a in CLI_ARGS]}
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "data.jsonl")
        with open(path, "w") as f:
            f.write("\n".join(cli_dataset_lines()) + "\n")
        tr, ev, he = ut._load_dataset(path, 8)
    out["dataset"] = {"train": [s["id"] for s in tr], "eval": [s["id"] for s in ev],
                      "heldout": [s["id"] for s in he]}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default=None, help="comma list of fixtures to (re)write")
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    torch.set_num_threads(os.cpu_count())
    only = set(a.only.split(",")) if a.only else None

    def want(name):
        return only is None or name in only
    if want("c1"):
        torch.save(run_case(a.reference, C1), os.path.join(HERE, "c1.pt"))
    if want("bf16_mini"):
        mini = dict(H=512, E=16, k=4, I=256, T=48, dtype=torch.bfloat16, seed=1, order="c2")
        torch.save(run_case(a.reference, mini), os.path.join(HERE, "bf16_mini.pt"))
    if want("router_ties"):
        torch.save(run_ties(a.reference), os.path.join(HERE, "router_ties.pt"))
    if want("rigl"):
        torch.save(run_rigl(a.reference), os.path.join(HERE, "rigl.pt"))
    if want("cli"):
        import json
        with open(os.path.join(HERE, "cli.json"), "w") as f:
            json.dump(run_cli(a.reference), f, indent=1)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
