"""Host logic of SparseTrainer's expert-parallel branch on CPU (gloo, 2 ranks).

* Selection: every rank's candidates of a full [E, R, C] tensor go through
  ``global_select``; the ranks get the same global list, equal to the
  single-process per-tensor top-k over the union of the candidates
  (usaf/moe_loader.py:613-628), and ``shard_share`` splits it into disjoint
  per-shard lists that together are that selection.  The device top-k is
  replaced by its CPU statement (descending score, ties to the lowest flat
  index) so that only the host logic runs.
* Decisions: ``ranks_agree`` makes one rank's non-finite shard skip the step
  on every rank, one rank's error word raise on every rank, and the logged
  loss the ranks' mean.
"""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cpu_select(vals, idxs, k):
    order = sorted(range(vals.numel()), key=lambda i: (-float(vals[i]), int(idxs[i])))[:k]
    return idxs[torch.tensor(order, dtype=torch.long)]


def _candidates(rank, El, numel_e):
    """Per-expert candidates of this rank's experts, with ties across ranks."""
    g = torch.Generator().manual_seed(40 + rank)
    vals, idxs = [], []
    for e in range(rank * El, (rank + 1) * El):
        loc = torch.randperm(numel_e, generator=g)[:30]
        v = torch.randint(0, 20, (30,), generator=g).float()   # many equal scores
        vals.append(v)
        idxs.append(loc + e * numel_e)
    return torch.cat(vals), torch.cat(idxs)


def _worker(rank, world, port, q):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        from usaf_b200 import expert_parallel, trainer
        expert_parallel.select_candidates = _cpu_select
        E, R, C = 4, 8, 16
        El, numel_e = E // world, R * C
        vals, idxs = _candidates(rank, El, numel_e)
        k = 25
        g = expert_parallel.global_select(vals, idxs, k)
        allv = torch.cat([_candidates(r, El, numel_e)[0] for r in range(world)])
        alli = torch.cat([_candidates(r, El, numel_e)[1] for r in range(world)])
        assert torch.equal(g, _cpu_select(allv, alli, k)), "global selection differs"
        span = El * numel_e
        share = trainer.shard_share(g, rank, span)
        assert share.numel() == 0 or (int(share.min()) >= 0 and int(share.max()) < span)
        shares = [torch.zeros(k, dtype=torch.long) for _ in range(world)]
        n = torch.tensor([share.numel()])
        ns = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(ns, n)
        padded = torch.full((k,), -1, dtype=torch.long)
        padded[: share.numel()] = share + rank * span
        dist.all_gather(shares, padded)
        union = torch.cat([s[: int(c)] for s, c in zip(shares, ns)])
        assert sorted(union.tolist()) == sorted(g.tolist()), "shares do not partition the selection"

        # decisions: flags (1 = finite), loss, error words
        nf = 2
        flags = [1.0, 0.0] if rank == 0 else [1.0, 1.0]
        out = trainer.ranks_agree(torch.tensor(flags + [2.0 + 2 * rank, 0.0]), nf)
        assert out[:nf].tolist() == [1.0, 0.0], out
        assert abs(float(out[nf]) - 3.0) < 1e-6 and float(out[nf + 1]) == 0.0
        errs = [0.0, 0.0] if rank == 0 else [0.0, 8.0]
        out = trainer.ranks_agree(torch.tensor([1.0, 1.0, 1.0] + errs), nf)
        assert out[:nf].tolist() == [1.0, 1.0] and float(out[nf + 1:].sum()) == 1.0, out
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


def test_trainer_expert_parallel_host_logic():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    world = 2
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res
