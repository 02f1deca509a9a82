"""Benchmark: sparse training step of a Qwen3-30B-A3B-shaped MoE layer.

One step = router + dispatch + grouped int4 SwiGLU GEMMs + combine (forward),
the full backward (combine, router, both dX GEMMs, dX gather), expert-weight
gradients at the 0.5% selected coordinates, and the SparseAdam updates of the
expert masters (with the overlay write-back) and of the full router.
Workload: T=4096 tokens, H=2048, E=128 experts, top-8,
I=768, bf16 activations, int4 group-128 experts; synthetic seeded data.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N>1 runs under torchrun, expert-parallel: every rank routes its own 4096
tokens, owns E/N experts (int4 weights, overlay, masters, Adam state), and
NCCL all-to-alls move the routed rows to the owners and back; the router
gradient is all-reduced (weak scaling: tokens per rank fixed).  value = all
ranks' tokens / max-over-ranks step time.
``--impl reference`` times the CPU restatement of the reference's own path
on the host cores, on rank 0 only: its batched dispatch
(benchmarks/kaggle_t4_bench.py:284-328, the reported value) next to the
dense-masked loop that train.py runs (usaf/qwen3moe_dml.py:24-86) and the
SGD-momentum router variant, each with capture and SparseAdam.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CFG = dict(T=4096, H=2048, E=128, k=8, I=768, frac=0.005, lr=1e-4)
# DRAM bytes (read + write) of one gate_up launch on this workload, from ncu
GATE_UP_DRAM_BYTES = 372.5e6 + 127.5e6


def gate_up_bytes(n_pairs: int) -> float:
    """Algorithmic bytes of one gate_up launch: int4 codes + fp16 scales and
    zeros of all experts, x_perm read, gu and h written (bf16)."""
    E, H, I = CFG["E"], CFG["H"], CFG["I"]
    w = E * 2 * I * H
    return w / 2 + w / 128 * 4 + n_pairs * H * 2 + n_pairs * 2 * I * 2 + n_pairs * I * 2
METRIC = "training tokens/s per step (Qwen3-30B-A3B-shape, int4, 0.5% sparse)"
UNIT = "tokens/s"


def peaks():
    """(HBM GB/s, bf16 TFLOP/s burst, bf16 TFLOP/s sustained, source) from
    MEASURED_PEAKS.json, else the pool's fallback figures."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return (float(p["hbm_gbs"]), float(p["bf16_tflops"]),
                float(p.get("bf16_tflops_sustained", p["bf16_tflops"])), "measured (MEASURED_PEAKS.json)")
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling (every 100 ms, with timestamps);
    :meth:`summary` keeps the samples taken inside the marked timed window."""

    FIELDS = ("timestamp,clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        # raw samples: $USAF_CLOCKS_DIR (to keep them) or the temp directory
        out_dir = os.environ.get("USAF_CLOCKS_DIR") or tempfile.gettempdir()
        self.path = os.path.join(out_dir, f"clocks_gpu{gpu}.csv")
        self.t0 = self.t1 = None

    def __enter__(self):
        try:
            os.makedirs(os.path.dirname(self.path), exist_ok=True)
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.5)   # let the sampler start before the timed window opens
        except Exception:
            self.proc = None
        return self

    def mark_start(self):
        self.t0 = time.time()

    def mark_end(self):
        self.t1 = time.time()

    def __exit__(self, *a):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        import datetime
        try:
            rows = []
            for line in open(self.path).read().strip().splitlines():
                r = [x.strip() for x in line.split(",")]
                if len(r) < 7:
                    continue
                try:
                    ts = datetime.datetime.strptime(r[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    continue
                rows.append((ts, r[1:]))
            win = [r for ts, r in rows if self.t0 is not None and self.t0 - 0.05 <= ts <= self.t1 + 0.05]
            sm = [float(r[0]) for r in win if r[0].replace(".", "").isdigit()]
            mx = float(win[0][1]) if win else (float(rows[0][1][1]) if rows else None)
            names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
            reasons = sorted({names[i] for r in win for i in range(4)
                              if r[2 + i] == "Active"})
            return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                    "reasons": reasons, "samples": len(sm)}
        except Exception as e:  # noqa: BLE001
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "error": str(e)[:80]}


# ------------------------------------------------------------------ ours ---
def build_layer(dev, seed: int):
    from usaf_b200.engine import Projection
    from usaf_b200.layer import SparseMoELayer
    from usaf_b200.quantization import quantize_4bit
    T, H, E, k, I = CFG["T"], CFG["H"], CFG["E"], CFG["k"], CFG["I"]
    g = torch.Generator(device=dev).manual_seed(seed)
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    w_r = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    projs = {}
    for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = torch.randn(*shape, device=dev, generator=g) * 0.02
        q, s, z, _ = quantize_4bit(w, 128)
        del w
        projs[n] = Projection(q, s, z, shape, 128, torch.bfloat16)
    dy = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    layer = SparseMoELayer(w_r, projs["gate_up_proj"], projs["down_proj"], k, T)
    store = layer.importance(x, dy, CFG["frac"])
    layer.init_selection(store.select(CFG["frac"]), lr=CFG["lr"])
    torch.cuda.synchronize()
    return layer, x, dy


def build_ep_layer(dev, rank: int, world: int):
    """Expert-parallel layer: the same model on every rank (seed 1), this
    rank's El = E/world experts, this rank's own token batch (seed 1+rank);
    importance-selected 0.5 % chosen globally across the shards."""
    from usaf_b200.engine import Projection
    from usaf_b200.expert_parallel import ExpertParallelLayer
    from usaf_b200.quantization import quantize_4bit
    T, H, E, k, I = CFG["T"], CFG["H"], CFG["E"], CFG["k"], CFG["I"]
    El, e0 = E // world, rank * (E // world)
    g = torch.Generator(device=dev).manual_seed(1)
    w_r = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    projs = {}
    for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = torch.randn(*shape, device=dev, generator=g) * 0.02
        q, s, z, _ = quantize_4bit(w[e0:e0 + El].contiguous(), 128)
        del w
        projs[n] = Projection(q, s, z, (El,) + shape[1:], 128, torch.bfloat16)
    gt = torch.Generator(device=dev).manual_seed(1 + rank)
    x = torch.randn(T, H, device=dev, generator=gt).to(torch.bfloat16)
    dy = torch.randn(T, H, device=dev, generator=gt).to(torch.bfloat16)
    layer = ExpertParallelLayer(w_r, projs["gate_up_proj"], projs["down_proj"], k, T)
    active = layer.importance(x, dy, CFG["frac"])
    layer.init_selection(active, lr=CFG["lr"])
    torch.cuda.synchronize()
    return layer, x, dy


def run_ours(args, rank, world, local_rank):
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    import usaf_b200  # noqa: F401
    from usaf_b200 import _lib
    import usaf_b200.expert_parallel as epm
    if world > 1:
        layer, x, dy = build_ep_layer(dev, rank, world)
        blk = layer.moe
    else:
        layer, x, dy = build_layer(dev, 1 + rank)
        blk = layer.block
    # the importance pass's dense |grad| buffers are gone: return their memory
    torch.cuda.empty_cache()
    T = CFG["T"]
    # timed kernel: the grouped gate_up dequant GEMM (+SwiGLU) of the forward
    k_ev = []
    orig_call = _lib.call

    def step(xs, dys):
        # NVTX range per step: lets a profiler capture exactly one step's launches
        torch.cuda.nvtx.range_push("usaf_step")
        out = layer.train_step(xs, dys)
        torch.cuda.nvtx.range_pop()
        return out

    for _ in range(args.warmup):
        step(x, dy)
    torch.cuda.synchronize()
    blk.check()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    # the router trains every step and the routing drifts with it (the number of
    # routed pairs grows as bf16 logits tie); both timed phases start from this state
    n_pairs_start = blk.n_rows_host() if world > 1 else blk.n_pairs_host()
    router_snap = (layer.w_r.detach().clone(), layer.router_opt.state_dict())

    def restore_router():
        layer.w_r.copy_(router_snap[0])
        layer.router_opt.load_state_dict(router_snap[1])
        torch.cuda.synchronize()

    rows_dev = blk.own_n if world > 1 else blk.n_pairs      # slots the gate_up launch processes
    k_rows = []

    def timed_call(name, *a):
        if name == "usaf_expert_gate_up_fwd":
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            orig_call(name, *a)
            e1.record()
            k_ev.append((e0, e1))
            k_rows.append(rows_dev.clone())     # device copy, read after the timed loop
        else:
            orig_call(name, *a)

    import usaf_b200.engine as eng
    eng.call = timed_call
    epm.call = timed_call
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        torch.cuda.synchronize()
        clk.mark_start()
        start.record()
        for _ in range(args.steps):
            step(x, dy)
        end.record()
        torch.cuda.synchronize()
        clk.mark_end()
    eng.call = orig_call
    epm.call = orig_call
    blk.check()
    ms = start.elapsed_time(end) / args.steps
    kern_ms = statistics.mean(a.elapsed_time(b) for a, b in k_ev)
    # slots the timed gate_up kernel processes on this rank (owner rows under EP)
    n_pairs = blk.n_rows_host() if world > 1 else blk.n_pairs_host()

    # end-to-end: a training loop through the public API with host buffers.  Every
    # step copies its inputs from pinned host memory and reads its scalar result
    # (sum(y * dy)) back to the host.  The copy of step i+1's inputs runs on a
    # second stream while step i computes (two device input buffers), and step
    # i's result is read once step i+1 has been queued.
    xh = x.cpu().pin_memory()
    dyh = dy.cpu().pin_memory()
    xd = [torch.empty_like(x) for _ in range(2)]
    dyd = [torch.empty_like(dy) for _ in range(2)]
    loss = [torch.empty(1, device=dev) for _ in range(2)]
    lossh = [torch.empty(1).pin_memory() for _ in range(2)]
    copy_stream = torch.cuda.Stream(device=dev)
    ev_copied = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]
    results = []
    copy_ev = []        # (start, end) of each step's input copy, timed loop only

    def issue_copy(i):
        b = i % 2
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(ev_used[b])          # step i-2 is done with buffer b
            if copy_ev is not None:
                c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                c0.record(copy_stream)
            xd[b].copy_(xh, non_blocking=True)
            dyd[b].copy_(dyh, non_blocking=True)
            if copy_ev is not None:
                c1.record(copy_stream)
                copy_ev.append((c0, c1))
            ev_copied[b].record(copy_stream)

    def run_step(i):
        b = i % 2
        cur = torch.cuda.current_stream()
        cur.wait_event(ev_copied[b])
        y, _, _ = layer.train_step(xd[b], dyd[b])
        _lib.call("usaf_dot", _lib.ptr(y), _lib.ptr(dyd[b]), _lib.BF16, y.numel(), _lib.ptr(loss[b]),
                  _lib.stream())
        lossh[b].copy_(loss[b], non_blocking=True)
        ev_used[b].record(cur)

    def e2e_loop(n):
        issue_copy(0)
        for i in range(n):
            issue_copy(i + 1)
            run_step(i)
            if i > 0:
                ev_used[(i - 1) % 2].synchronize()
                results.append(float(lossh[(i - 1) % 2].item()))
        ev_used[(n - 1) % 2].synchronize()
        results.append(float(lossh[(n - 1) % 2].item()))
        torch.cuda.current_stream().wait_stream(copy_stream)   # the spare prefetch

    e2e_loop(2)
    torch.cuda.synchronize()
    copy_ev.clear()
    restore_router()
    if world > 1:
        torch.distributed.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    copy_stream.wait_event(e0)      # the first input copy starts inside the timed window
    e2e_loop(args.steps)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / args.steps
    # the input copies of the timed steps (the last one prefetches a step that is not run)
    h2d_ms = statistics.mean(a.elapsed_time(b) for a, b in copy_ev[:args.steps])

    hbm, burst, sustained, src = peaks()
    H, I = CFG["H"], CFG["I"]
    # FLOPs of the mean launch: routed slots averaged over the timed launches
    mean_rows = float(torch.stack(k_rows).double().mean().item())
    flops = 2.0 * mean_rows * (2 * I) * H
    achieved = flops / (kern_ms * 1e-3) / 1e12
    if world > 1:
        t = torch.tensor([ms, e2e_ms, kern_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms, e2e_ms, kern_ms = t.tolist()
        a = torch.tensor([achieved], device=dev)      # the slowest rank's kernel rate
        torch.distributed.all_reduce(a, op=torch.distributed.ReduceOp.MIN)
        achieved = float(a.item())
    # the kernel is timed inside a short window: the burst GEMM peak is its
    # denominator unless the clocks sampled in the window show the power cap
    clk_sum = clk.summary()
    capped = "sw_power_cap" in (clk_sum.get("reasons") or [])
    tflops = sustained if capped else burst
    peak_src = f"{src}, bf16 {'sustained (sw_power_cap seen)' if capped else 'burst (no power cap in the window)'}"
    launches, lib_launches = count_launches(lambda: step(x, dy))
    variants = {}
    if world == 1:
        # train.py's router optimizer (SGD, momentum 0.9, train.py:494-498) in place of
        # SparseAdam over W_r; the rest of the step unchanged, same starting router state
        layer.w_r.copy_(router_snap[0])
        layer.use_router_optimizer("sgd", CFG["lr"])
        for _ in range(args.warmup):
            step(x, dy)
        v0 = torch.cuda.Event(enable_timing=True)
        v1 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        v0.record()
        for _ in range(args.steps):
            step(x, dy)
        v1.record()
        torch.cuda.synchronize()
        blk.check()
        sgd_ms = v0.elapsed_time(v1) / args.steps
        variants["router_sgd"] = {"value": T / (sgd_ms * 1e-3), "unit": UNIT, "ms_per_step": sgd_ms,
                                  "router": "SGD momentum 0.9 (train.py:494-498)"}
        layer.w_r.copy_(router_snap[0])
        layer.use_router_optimizer("adam", CFG["lr"])
    out = {
        "metric": METRIC, "value": world * T / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) tokens, N(0,0.02) weights quantized to int4 g128)",
        "config": {"workload": "C2: one Qwen3-30B-A3B MoE layer, fwd+bwd+sparse grads+SparseAdam",
                   "T": T, "H": H, "E": CFG["E"], "top_k": CFG["k"], "I": I, "active_frac": CFG["frac"],
                   "routed_pairs": n_pairs, "routed_pairs_at_start": n_pairs_start,
                   "parallelism": f"ep{world} (experts sharded, NCCL all-to-all)" if world > 1 else "single",
                   "l2": "working set (~1.5 GB int4 weights + activations) exceeds the 126 MB L2"},
        "e2e": {"value": world * T / (e2e_ms * 1e-3), "unit": UNIT,
                "h2d_bytes_per_step": x.numel() * 2 + dy.numel() * 2, "d2h_bytes_per_step": 4,
                "ms_per_step": e2e_ms, "h2d_ms_per_step": h2d_ms,
                "h2d_gbps": (x.numel() * 2 + dy.numel() * 2) / (h2d_ms * 1e-3) / 1e9},
        "roofline": {"bound": "tensor", "kernel": "usaf_expert_gate_up_fwd (grouped int4 GEMM + SwiGLU)",
                     "achieved": achieved, "peak": tflops, "unit": "TFLOP/s",
                     "frac": achieved / tflops, "peak_source": peak_src,
                     "frac_of_sustained": achieved / sustained, "kernel_ms": kern_ms,
                     "slots_per_launch": mean_rows,
                     "traffic": GATE_UP_DRAM_BYTES if world == 1 else None,
                     "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                       "launch of this kernel on this workload (--set full capture)",
                     "algorithmic_bytes": gate_up_bytes(mean_rows)},
        "variants": variants,
        "gpu_launches": launches * args.steps,
        "launches_per_step": {"usaf_b200": launches, "torch_and_copies": lib_launches},
        "clocks": clk_sum,
    }
    return out


def count_launches(step_fn):
    """Kernels launched by one step, counted by the CUDA profiler (CUPTI)
    outside the timed region: (this library's kernels, everything else --
    torch's fills/copies and NCCL's collectives).  A library kernel is any
    kernel whose name is not torch's (at::), NCCL's or a memcpy/memset."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step_fn()
        torch.cuda.synchronize()
    ours = other = 0
    for ev in prof.events():
        if str(ev.device_type) != "DeviceType.CUDA":
            continue
        n = ev.name
        if (n.startswith("Memcpy") or n.startswith("Memset") or "at::" in n or "cub::" in n
                or "nccl" in n.lower()):
            other += 1
        else:
            ours += 1
    return ours, other


# ------------------------------------------------------------- reference ---
_CPU_LAYER = []


def _cpu_layer():
    """The C2 layer for the CPU reference path, built once per process:
    router, int4-quantized experts dequantized to bf16 (the reference's
    fp16 -> compute-dtype weights), a 0.5 % active set."""
    if not _CPU_LAYER:
        import numpy as np
        from oracle import quant as oquant
        H, E, I = CFG["H"], CFG["E"], CFG["I"]
        torch.manual_seed(1)
        w_r = (torch.randn(E, H) * 0.02).to(torch.bfloat16)
        dense, active, shapes = [], {}, {}
        gen = np.random.default_rng(0)
        for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
            w = (torch.randn(*shape) * 0.02).numpy()
            q, s, z, _ = oquant.quantize_4bit(w, 128)
            del w
            d = oquant.dequantize_4bit(q, s, z, shape, 128)
            dense.append(torch.from_numpy(d).to(torch.bfloat16))
            numel = int(np.prod(shape))
            name = f"layer.mlp.experts.{n}"
            active[name] = torch.from_numpy(gen.choice(numel, int(numel * CFG["frac"]), replace=False))
            shapes[name] = shape
        _CPU_LAYER.append((w_r, dense, active, shapes))
    return _CPU_LAYER[0]


def run_reference_cpu(sample_tokens: int, iters: int, experts: str = "batched",
                      router: str = "adam"):
    """Time the oracle restatement of the reference's CPU path on the host
    cores: one C2-shaped layer's forward and backward with SparseGradStore
    capture, then SparseAdam over the masters and a router step.

    ``experts``: ``"batched"`` is the reference's batched dispatch
    (benchmarks/kaggle_t4_bench.py:284-328: tokens grouped by expert into a
    padded batch, two bmm), its fastest CPU path; ``"dense"`` the
    dense-masked loop that train.py runs (usaf/qwen3moe_dml.py:24-64: every
    expert on every token).  ``router``: ``"adam"`` SparseAdam over all of
    W_r (the C2 configuration), ``"sgd"`` train.py's SGD with momentum
    (train.py:494-498).  Returns (tokens/s, seconds per step): the median of
    ``iters`` steps after one warm-up step."""
    from oracle import moe as omoe
    torch.set_num_threads(os.cpu_count())
    T, H, E, k, I = sample_tokens, CFG["H"], CFG["E"], CFG["k"], CFG["I"]
    w_r, dense, active, shapes = _cpu_layer()
    g = torch.Generator().manual_seed(1)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    dy = torch.randn(T, H, generator=g).to(torch.bfloat16)
    masters = {n: dense[i].float().reshape(-1)[active[n]].clone()
               for i, n in enumerate(shapes)}
    opt = omoe.SparseAdam({n: masters[n] for n in shapes}, active, compact_params=True)
    w_r_p = torch.nn.Parameter(w_r.clone(), requires_grad=False)
    if router == "sgd":
        ropt = torch.optim.SGD([w_r_p], lr=CFG["lr"], momentum=0.9, weight_decay=0.01)
    else:
        ropt = omoe.SparseAdam({"r": w_r_p.data}, {"r": torch.arange(E * H)})
    times = []
    for it in range(iters + 1):
        t0 = time.perf_counter()
        store = omoe.SparseGradStore(active, shapes)
        res = omoe.block_step(x, w_r_p.data, dense[0], dense[1], dy, k, True, capture=store.add,
                              prefix="layer.mlp.experts", experts=experts)
        opt.step(store.compact)
        if router == "sgd":
            w_r_p.grad = res["dW_r"]
            ropt.step()
            w_r_p.grad = None
        else:
            ropt.step({"r": res["dW_r"]})
        times.append(time.perf_counter() - t0)
    med = statistics.median(times[1:])
    return T / med, med


def reference_arm(iters: int, batched_tokens: int, dense_tokens: int) -> dict:
    """The reference's CPU path on this host, three ways: the batched dispatch
    (its fastest path; the reported value), the dense-masked loop train.py
    runs, and the batched path with train.py's SGD-momentum router."""
    vb, sb = run_reference_cpu(batched_tokens, iters, "batched", "adam")
    vd, sd = run_reference_cpu(dense_tokens, iters, "dense", "adam")
    vs, ss = run_reference_cpu(batched_tokens, iters, "batched", "sgd")
    return {"value": vb, "ms_per_step": sb * 1e3, "unit": UNIT, "cores": os.cpu_count(),
            "kind": "port", "cpu": cpu_info(),
            "sample": f"{batched_tokens} tokens of the C2 layer per step (batched dispatch, "
                      f"SparseAdam router), median of {iters} steps after 1 warm-up",
            "paths": {
                "batched_dispatch": {"tokens_per_s": vb, "ms_per_step": sb * 1e3,
                                     "sample_tokens": batched_tokens,
                                     "ref": "benchmarks/kaggle_t4_bench.py:284-328"},
                "dense_masked": {"tokens_per_s": vd, "ms_per_step": sd * 1e3,
                                 "sample_tokens": dense_tokens,
                                 "ref": "usaf/qwen3moe_dml.py:24-64 (train.py's path)"},
                "batched_router_sgd": {"tokens_per_s": vs, "ms_per_step": ss * 1e3,
                                       "sample_tokens": batched_tokens,
                                       "ref": "train.py:494-498 router optimizer"}}}


def run_c4_sweep(steps: int = 10):
    """forward and backward of one C2-shaped layer timed
    separately at T in {1, 16, 256, 4096, 16384}, uniform and Zipf(1.2)
    routing (biased router logits: constant feature x[:,0]=1 plus log p_e on
    w_r[:,0]), random 0.5% overlays; CUDA events, one JSON line per point."""
    from usaf_b200.engine import BlockDims, MoEBlock, Projection
    from usaf_b200.quantization import quantize_4bit
    dev = torch.device("cuda", 0)
    H, E, k, I = CFG["H"], CFG["E"], CFG["k"], CFG["I"]
    g = torch.Generator(device=dev).manual_seed(1)
    projs = {}
    for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = torch.randn(*shape, device=dev, generator=g) * 0.02
        q, s_, z, _ = quantize_4bit(w, 128)
        del w
        p = Projection(q, s_, z, shape, 128, torch.bfloat16)
        numel = p.numel()
        idx = torch.randperm(numel, device=dev, generator=g)[: int(numel * CFG["frac"])]
        p.set_overlay(idx, torch.randn(idx.numel(), device=dev, generator=g) * 0.02)
        projs[n] = p
    gu, dn = projs["gate_up_proj"], projs["down_proj"]
    hbm_peak, tc_peak, _, _ = peaks()
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    for routing in ("uniform", "zipf1.2"):
        for T in (1, 16, 256, 4096, 16384):
            x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
            dy = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
            w_r = torch.randn(E, H, device=dev, generator=g) * 0.02
            if routing != "uniform":
                x[:, 0] = 1.0
                pe = torch.arange(1, E + 1, device=dev, dtype=torch.float64) ** -1.2
                w_r[:, 0] += torch.log(pe / pe.sum()).float()
            w_r = w_r.to(torch.bfloat16)
            blk = MoEBlock(BlockDims(T, H, E, I, k, True, torch.bfloat16), dev)
            cg = torch.zeros(gu.n_ov, device=dev)
            cd = torch.zeros(dn.n_ov, device=dev)
            for _ in range(3):
                blk.forward(x, w_r, gu, dn)
                blk.backward(dy, x, w_r, gu, dn)
                blk.sparse_grads(gu, dn, cg, cd)
            torch.cuda.synchronize()
            a, b, c = ev(), ev(), ev()
            tf = tb = 0.0
            for _ in range(steps):
                a.record()
                blk.forward(x, w_r, gu, dn)
                b.record()
                blk.backward(dy, x, w_r, gu, dn)
                blk.sparse_grads(gu, dn, cg, cd)
                c.record()
                torch.cuda.synchronize()
                tf += a.elapsed_time(b)
                tb += b.elapsed_time(c)
            blk.check()
            P = blk.n_pairs_host()
            fwd_flop = 2.0 * P * 3 * I * H
            # HBM floor of the grouped GEMMs: the int4 codes + fp16 scale/zero of every
            # expert hit, read once per pass (gate_up + down forward; down_bwd + gate_up_bwd)
            hit = int((blk.expert_cnt > 0).sum().item())
            w_bytes = hit * 3 * I * H * (0.5 + 4.0 / 128)
            fwd_s, bwd_s = tf / steps * 1e-3, tb / steps * 1e-3
            print(json.dumps({"config": "C4", "routing": routing, "T": T, "pairs": P,
                              "fwd_ms": tf / steps, "bwd_ms": tb / steps,
                              "fwd_tflops": fwd_flop / fwd_s / 1e12,
                              "bwd_tflops": fwd_flop / bwd_s / 1e12,
                              "experts_hit": hit, "weight_mb_per_pass": w_bytes / 1e6,
                              "fwd_weight_gbps": w_bytes / fwd_s / 1e9,
                              "fwd_hbm_frac": w_bytes / fwd_s / 1e9 / hbm_peak,
                              "fwd_tensor_frac": fwd_flop / fwd_s / 1e12 / tc_peak,
                              "max_expert_tokens": int(blk.expert_cnt.max().item())}), flush=True)
            del blk


def run_importance(steps: int = 5, warmup: int = 2):
    """The importance pass of the C2 layer (one forward/backward, the per-expert
    top-``2*frac`` candidates of TopKImportanceStore and the per-tensor select;
    usaf/moe_loader.py:584-631, train.py:540-546), one GPU, CUDA events; one
    JSON line.  The candidates come from three tensor-core SDDMM passes that
    never write the gradient (exponent histogram, histogram inside the
    threshold bucket, emission); the line also times the dense path it
    replaces (fp32 |dW| buffer + per-expert radix top-k) on the same batch.
    Roofline: the dense products of a pass (2 P (2I H + H I) FLOP) over the
    pass's kernel time, against the burst bf16 peak."""
    from usaf_b200 import _lib
    import usaf_b200.engine as eng
    from usaf_b200.moe_loader import TopKImportanceStore
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    layer, x, dy = build_layer(dev, 1)
    torch.cuda.empty_cache()
    frac = CFG["frac"]
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def fused():
        store = layer.importance(x, dy, frac)
        return store.select(frac)

    def dense():
        layer.forward_backward(x, dy)
        store = TopKImportanceStore(layer.shapes, frac)
        for name in layer.names:
            which = name.rsplit(".", 1)[1]
            store.add_dense_abs(name, layer.block.dense_abs_grad(which), layer.block.hit_experts())
        return store.select(frac)

    def timed(fn, n):
        a, b = ev(), ev()
        torch.cuda.synchronize()
        a.record()
        for _ in range(n):
            out = fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n, out

    for _ in range(warmup):
        fused()
        dense()
    peak_mem0 = torch.cuda.memory_allocated()
    torch.cuda.reset_peak_memory_stats()
    fused_ms, sel_f = timed(fused, steps)
    fused_mem = torch.cuda.max_memory_allocated() - peak_mem0
    torch.cuda.reset_peak_memory_stats()
    dense_ms, sel_d = timed(dense, max(1, steps // 2))
    dense_mem = torch.cuda.max_memory_allocated() - peak_mem0
    same = all(torch.equal(sel_f[n], sel_d[n]) for n in sel_f)
    # kernel times of the SDDMM passes inside one fused pass
    orig = _lib.call
    kev = {}

    def hook(name, *a):
        if name in ("usaf_importance_hist", "usaf_importance_emit"):
            e0, e1 = ev(), ev()
            e0.record()
            orig(name, *a)
            e1.record()
            kev.setdefault(name, []).append((e0, e1))
        else:
            orig(name, *a)

    eng.call = hook
    fused()
    torch.cuda.synchronize()
    eng.call = orig
    hist_ms = sum(a.elapsed_time(b) for a, b in kev["usaf_importance_hist"])
    emit_ms = sum(a.elapsed_time(b) for a, b in kev["usaf_importance_emit"])
    P = layer.block.n_pairs_host()
    flop_pass = 2.0 * P * 3 * CFG["I"] * CFG["H"]
    _, tc_peak, _, src = peaks()
    per_pass_ms = (hist_ms + emit_ms) / 3
    print(json.dumps({"config": "C2", "mode": "importance",
                      "workload": "importance pass of one Qwen3-30B-A3B MoE layer (T 4096, top-8 candidates "
                                  "of 1 % per expert, select 0.5 % per tensor), int4 g128, bf16",
                      "fused_ms": fused_ms, "dense_path_ms": dense_ms,
                      "speedup_vs_dense_path": dense_ms / fused_ms,
                      "fused_extra_mem_gb": fused_mem / 1e9, "dense_path_extra_mem_gb": dense_mem / 1e9,
                      "same_selection_as_dense_path": same,
                      "sddmm_passes_ms": {"hist_two_passes": hist_ms, "emit": emit_ms},
                      "roofline": {"bound": "tensor", "achieved": flop_pass / (per_pass_ms * 1e-3) / 1e12,
                                   "peak": tc_peak, "unit": "TFLOP/s",
                                   "frac": flop_pass / (per_pass_ms * 1e-3) / 1e12 / tc_peak,
                                   "flop_per_pass": flop_pass, "peak_source": src},
                      "pairs": P, "steps": steps, "warmup": warmup, "data": "synthetic"}), flush=True)


def run_c5(steps: int = 10, warmup: int = 3):
    """BASELINE configs[4] on one GPU: a Mixtral-8x22B-shaped layer (H=6144,
    E=8, top-2, I=16384, T=4096, int4 g128 experts, bf16): one importance
    dense-gradient pass, selection of 0.5 %, then sparse training steps
    (SparseMoELayer.train_step), CUDA events; one JSON line."""
    from usaf_b200.engine import Projection
    from usaf_b200.layer import SparseMoELayer
    from usaf_b200.quantization import quantize_4bit
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    T, H, E, k, I, frac = 4096, 6144, 8, 2, 16384, 0.005
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    dy = torch.randn(T, H, device=dev, generator=g).to(torch.bfloat16)
    w_r = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    projs = {}
    for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
        w = torch.randn(*shape, device=dev, generator=g) * 0.02
        q, s_, z, _ = quantize_4bit(w, 128)
        del w
        projs[n] = Projection(q, s_, z, shape, 128, torch.bfloat16)
    layer = SparseMoELayer(w_r, projs["gate_up_proj"], projs["down_proj"], k, T)
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    layer.importance(x, dy, frac)                       # warm-up of the dense pass
    torch.cuda.synchronize()
    a, b = ev(), ev()
    a.record()
    store = layer.importance(x, dy, frac)
    active = store.select(frac)
    b.record()
    torch.cuda.synchronize()
    imp_ms = a.elapsed_time(b)
    layer.init_selection(active, lr=1e-4)
    for _ in range(warmup):
        layer.train_step(x, dy)
    torch.cuda.synchronize()
    a.record()
    for _ in range(steps):
        layer.train_step(x, dy)
    b.record()
    torch.cuda.synchronize()
    layer.block.check()
    ms = a.elapsed_time(b) / steps
    P = layer.block.n_pairs_host()
    flop = 2.0 * P * 3 * I * H * 2          # forward + dX backward of the grouped GEMMs
    print(json.dumps({"config": "C5", "workload": "one Mixtral-8x22B-shaped MoE layer (H 6144, E 8, top-2, "
                      "I 16384), int4 g128, bf16, T 4096", "importance_pass_ms": imp_ms,
                      "n_active": sum(a_.numel() for a_ in active.values()),
                      "step_ms": ms, "tokens_per_s": T / (ms * 1e-3), "pairs": P,
                      "grouped_gemm_tflops_per_step": flop / (ms * 1e-3) / 1e12,
                      "steps": steps, "warmup": warmup, "data": "synthetic"}), flush=True)


def run_c3(n_layers: int = 2, steps: int = 5, warmup: int = 2, recompute: bool = True):
    """BASELINE configs[2] (C3), on one GPU or, under torchrun, with the experts
    sharded over the ranks (each rank its own micro-batch): a random-init Qwen3MoeForCausalLM
    with the C3 shapes (H 2048, 32/4 heads, head dim 128, E 128, top-8, I 768,
    vocab 151936) at ``n_layers`` of its 48 layers, int4 g128 experts attached
    through patch_qwen3moe_for_b200, sequence 2048 x micro-batch 4, LM
    cross-entropy, trained by usaf_b200.trainer.SparseTrainer (importance
    pass, 0.5 % selection, loss scaling, SparseAdam + SGD-momentum router).
    Attention, norms, embeddings and the LM head run in PyTorch.  Memory for
    the full depth: the experts are built without dense weights, the blocks
    share their backward-only buffers, the pair buffers hold 1.25 x top_k
    pairs per token, and (``recompute``, as the reference's loader enables,
    usaf/moe_loader.py:758-760) each decoder layer's activations are
    recomputed in the backward.  One JSON line with the whole-model tokens/s."""
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeForCausalLM
    from usaf_b200 import qwen3moe
    from usaf_b200.engine import Projection
    from usaf_b200.quantization import quantize_4bit
    from usaf_b200.trainer import SparseTrainer
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    if world > 1:   # experts sharded over the ranks, every rank its own micro-batch
        torch.distributed.init_process_group(
            "nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=300))
    qwen3moe.patch_qwen3moe_for_b200()
    qwen3moe.configure_workspaces(pair_factor=1.25, share_backward=True)
    H, E, k, I, V, S, MB = 2048, 128, 8, 768, 151936, 2048, 4
    El, e0 = E // world, rank * (E // world)
    cfg = Qwen3MoeConfig(vocab_size=V, hidden_size=H, intermediate_size=6144, num_hidden_layers=n_layers,
                         num_attention_heads=32, num_key_value_heads=4, head_dim=128,
                         moe_intermediate_size=I, num_experts=E, num_experts_per_tok=k,
                         norm_topk_prob=True, max_position_embeddings=4096)
    torch.manual_seed(3)
    with torch.device(dev), qwen3moe.without_dense_experts():
        model = Qwen3MoeForCausalLM(cfg).to(torch.bfloat16)
    for p_ in model.parameters():
        p_.requires_grad_(False)
    if recompute:
        model.gradient_checkpointing_enable(gradient_checkpointing_kwargs={"use_reentrant": False})
    model.train()
    g = torch.Generator(device=dev).manual_seed(3)
    for layer in model.model.layers:
        mlp = layer.mlp
        mlp.gate.weight.requires_grad_(True)
        ps = []
        for shape in ((E, 2 * I, H), (E, H, I)):
            # the same full tensor on every rank (one generator stream); this rank keeps its shard
            rows = []
            for e in range(E):
                w_e = torch.randn(*shape[1:], device=dev, generator=g) * 0.02
                if e0 <= e < e0 + El:
                    rows.append(w_e)
            shard = torch.stack(rows)
            del rows
            q, s_, z, _ = quantize_4bit(shard, 128)
            del shard
            ps.append(Projection(q, s_, z, (El,) + shape[1:], 128, torch.bfloat16))
        qwen3moe.attach_int4_experts(mlp.experts, *ps, expert_parallel=world > 1)
    gt = torch.Generator(device=dev).manual_seed(4 + rank)
    batches = [torch.randint(0, V, (MB, S), device=dev, generator=gt) for _ in range(2)]
    lm = lambda m, ids: m(input_ids=ids, labels=ids).loss  # noqa: E731
    tr = SparseTrainer(model, steps=1000, lr_peak=2e-4, accum=1, frac=0.005, reselect_every=10 ** 9)
    tr.init_selection(tr.importance(batches[0], lm))
    for i in range(warmup):
        tr.train_step([batches[i % 2]], lm)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    logs = [tr.train_step([batches[i % 2]], lm) for i in range(steps)]
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / steps
    if world > 1:   # the slowest rank's time (CUDA events), whole-job tokens
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank != 0:
        return
    print(json.dumps({"config": "C3", "workload": f"Qwen3-30B-A3B-shaped causal LM, {n_layers} of 48 layers "
                      "(C3 layer shapes), seq 2048 x mb 4 per GPU, LM cross-entropy, int4 experts, 0.5% "
                      "sparse, SparseTrainer steps", "layers": n_layers, "n_gpus": world,
                      "parallelism": f"ep{world}" if world > 1 else "single",
                      "tokens_per_step": world * MB * S,
                      "step_ms": ms, "tokens_per_s": world * MB * S / (ms * 1e-3),
                      "ms_per_layer_incl_head": ms / n_layers, "activation_recompute": recompute,
                      "max_memory_gb": torch.cuda.max_memory_allocated(dev) / 1e9,
                      "losses": [round(l_["loss"], 4) for l_ in logs],
                      "all_finite": all(l_["finite"] for l_ in logs), "steps": steps, "warmup": warmup,
                      "data": "synthetic (uniform token ids)"}), flush=True)


def cpu_info():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-sample-tokens", type=int, default=192,
                    help="tokens per step of the dense-masked CPU reference path")
    ap.add_argument("--cpu-batched-tokens", type=int, default=1024,
                    help="tokens per step of the batched-dispatch CPU reference path")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--c4-sweep", action="store_true",
                    help="time forward and backward separately over the C4 token sweep (1 GPU)")
    ap.add_argument("--importance", action="store_true",
                    help="C2 importance pass, fused vs the dense |grad| path (1 GPU)")
    ap.add_argument("--c5", action="store_true",
                    help="Mixtral-8x22B-shaped layer: importance pass + sparse steps (1 GPU)")
    ap.add_argument("--c3", type=int, default=0, metavar="LAYERS",
                    help="C3-shaped causal LM with this many layers through SparseTrainer (1 GPU)")
    ap.add_argument("--c3-no-recompute", action="store_true",
                    help="keep every decoder layer's activations instead of recomputing them")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    if args.c4_sweep:
        run_c4_sweep()
        return
    if args.importance:
        run_importance()
        return
    if args.c5:
        run_c5()
        return
    if args.c3:
        run_c3(args.c3, recompute=not args.c3_no_recompute)
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        iters = max(1, min(args.steps, 3))
        ref = reference_arm(iters, args.cpu_batched_tokens, args.cpu_sample_tokens)
        v = ref["value"]
        out = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": iters,
               "warmup": 1, "ms_per_step": ref["ms_per_step"], "higher_is_better": True,
               "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
               "impl": "reference",
               "config": {"workload": "C2 layer shapes, the reference's batched-dispatch CPU path "
                                      "on host cores",
                          "T_sample": args.cpu_batched_tokens},
               "cpu_baseline": ref,
               "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(out))
        return

    if world > 1:
        torch.distributed.init_process_group(
            "nccl", device_id=torch.device("cuda", local_rank),
            timeout=__import__("datetime").timedelta(seconds=120))
    out = run_ours(args, rank, world, local_rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = reference_arm(1, args.cpu_batched_tokens, args.cpu_sample_tokens)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(out))


if __name__ == "__main__":
    main()
