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


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    a = ap.parse_args()
    sys.path.insert(0, a.reference)
    torch.set_num_threads(os.cpu_count())
    torch.save(run_case(a.reference, C1), os.path.join(HERE, "c1.pt"))
    mini = dict(H=512, E=16, k=4, I=256, T=48, dtype=torch.bfloat16, seed=1, order="c2")
    torch.save(run_case(a.reference, mini), os.path.join(HERE, "bf16_mini.pt"))
    torch.save(run_ties(a.reference), os.path.join(HERE, "router_ties.pt"))
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
