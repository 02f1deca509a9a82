"""Expert parallelism on the GPU.

* usaf_ep_permute against the reference index arithmetic (one GPU).
* Two ranks over NCCL (needs two GPUs): every rank routes its own tokens,
  owns half of the experts, and the results must equal one process running
  the whole batch (the ranks' token batches concatenated) with all experts:
  y and dX bit-for-bit per token (same routing, same per-expert slot order,
  same kernels), compact expert gradients of the rank's experts bit-for-bit,
  the router gradient within bf16 tolerance (rel <= 2e-2: the ranks' bf16
  partial gradients are summed in fp32 instead of one fp32 accumulation).
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_permute_kernel_vs_reference():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import sys
    sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
    import ep_reference
    from usaf_b200.expert_parallel import device_permute
    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(1)
    for W, El, H in ((2, 8, 64), (4, 4, 2048), (8, 16, 768), (1, 3, 8)):
        counts = torch.randint(0, 40, (W, El), generator=g, dtype=torch.int32)
        counts[0, 0] = 0
        n = int(counts.sum())
        rows = torch.randn(n, H, generator=g).to(torch.bfloat16)
        ref = torch.empty_like(rows)
        ep_reference.permute(counts, rows, ref, False)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        out = torch.empty(n, H, dtype=torch.bfloat16, device=dev)
        cd = counts.to(dev)
        device_permute(cd, rows.to(dev), out, False, err)
        back = torch.empty_like(out)
        device_permute(cd, out, back, True, err)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(out.cpu(), ref), (W, El, H)
        assert torch.equal(back.cpu(), rows), (W, El, H)


def _ep_worker(rank, world, port, q):
    try:
        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, device_id=dev)
        from usaf_b200.engine import BlockDims, MoEBlock, Projection
        from usaf_b200.expert_parallel import ExpertParallelMoE
        from usaf_b200.quantization import quantize_4bit
        T, H, E, k, I = 256, 512, 16, 4, 256
        El = E // world
        g = torch.Generator(device=dev).manual_seed(5)     # same model on every rank
        w_r = torch.randn(E, H, device=dev, generator=g) * 0.02
        x_all = torch.randn(world * T, H, device=dev, generator=g).to(torch.bfloat16)
        x_all[:, 0] = 1.0
        p = torch.arange(1, E + 1, device=dev, dtype=torch.float64) ** -1.2
        w_r[:, 0] += torch.log(p / p.sum()).float()        # skewed routing
        w_r = w_r.to(torch.bfloat16)
        dy_all = torch.randn(world * T, H, device=dev, generator=g).to(torch.bfloat16)
        full, loc = {}, {}
        for n, shape in (("gate_up_proj", (E, 2 * I, H)), ("down_proj", (E, H, I))):
            w = torch.randn(*shape, device=dev, generator=g) * 0.02
            qq, ss, zz, _ = quantize_4bit(w, 128)
            numel = w.numel()
            idx = torch.randperm(numel, device=dev, generator=g)[: int(numel * 0.005)]
            master = torch.randn(idx.numel(), device=dev, generator=g) * 0.02
            pf = Projection(qq, ss, zz, shape, 128, torch.bfloat16)
            pf.set_overlay(idx, master)
            ne = shape[1] * shape[2]
            e0 = rank * El
            qf, sf, zf = qq.reshape(-1), ss.reshape(-1), zz.reshape(-1)
            pl = Projection(qf[e0 * ne // 2:(e0 + El) * ne // 2].clone(),
                            sf[e0 * ne // 128:(e0 + El) * ne // 128].clone(),
                            zf[e0 * ne // 128:(e0 + El) * ne // 128].clone(),
                            (El,) + shape[1:], 128, torch.bfloat16)
            mine = (idx >= e0 * ne) & (idx < (e0 + El) * ne)
            pl.set_overlay(idx[mine] - e0 * ne, master[mine])
            full[n], loc[n] = (pf, mine), pl
        # one process, whole batch, all experts
        ref = MoEBlock(BlockDims(world * T, H, E, I, k, True, torch.bfloat16), dev)
        y_ref = ref.forward(x_all, w_r, full["gate_up_proj"][0], full["down_proj"][0]).clone()
        dx_ref, dwr_ref = ref.backward(dy_all, x_all, w_r, full["gate_up_proj"][0], full["down_proj"][0])
        cg = {n: torch.zeros(full[n][0].n_ov, device=dev) for n in full}
        ref.sparse_grads(full["gate_up_proj"][0], full["down_proj"][0], cg["gate_up_proj"], cg["down_proj"])
        ref.check()
        # expert parallel, this rank's tokens
        sl = slice(rank * T, (rank + 1) * T)
        ep = ExpertParallelMoE(w_r, loc["gate_up_proj"], loc["down_proj"], k, T)
        y = ep.forward(x_all[sl].contiguous(), w_r).clone()
        ce = {n: torch.zeros(loc[n].n_ov, device=dev) for n in loc}
        # expert gradients computed while the dX rows travel back (the training path)
        dx, dw_r = ep.backward(dy_all[sl].contiguous(), x_all[sl].contiguous(), w_r,
                               compact_gu=ce["gate_up_proj"], compact_dn=ce["down_proj"])
        torch.cuda.synchronize()
        ep.check()
        assert torch.equal(y, y_ref[sl]), "y"
        assert torch.equal(dx, dx_ref[sl]), "dX"
        rel = ((dw_r.double() - dwr_ref.double()).norm() / dwr_ref.double().norm()).item()
        assert rel <= 2e-2, f"dW_r rel {rel}"
        for n in full:
            assert torch.equal(ce[n], cg[n][full[n][1]]), f"compact {n}"
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        import traceback
        q.put((rank, repr(e) + traceback.format_exc()[-800:]))


def test_expert_parallel_two_ranks_vs_one_process():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
    assert all(v == "ok" for v in res.values()), res
