"""Host logic of expert parallelism on CPU with the gloo backend (world size
2, 3 and 4, and a rank that routes no rows at all): count exchange, split
sizes, the all-to-all of rows to the experts' owners in expert-major order
and the way back.  The regrouping uses the
reference index arithmetic of tests/ep_reference.py (the device kernel is
checked against the same arithmetic in tests/test_gpu_ep.py)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, E, H, q, empty_rank=-1):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world)
        import sys
        sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
        import ep_reference
        from usaf_b200.expert_parallel import ExpertExchange
        El = E // world
        g = torch.Generator().manual_seed(100 + rank)
        cnt = torch.randint(0, 6, (E,), generator=g, dtype=torch.int32)
        cnt[rank] = 0                                   # an expert without rows
        if rank == empty_rank:
            cnt.zero_()                                 # this rank routes nothing
        # expert-major rows of this rank: value = (rank, expert, index, column)
        rows = []
        for e in range(E):
            for i in range(int(cnt[e])):
                rows.append([rank * 1e6 + e * 1e3 + i + c * 1e-3 for c in range(H)])
        src = torch.tensor(rows, dtype=torch.float64).reshape(-1, H)
        ex = ExpertExchange(E, permute=ep_reference.permute)
        xp = ex.plan(cnt)
        # every rank's counts, to know what to expect
        allc = [torch.zeros_like(cnt) for _ in range(world)]
        dist.all_gather(allc, cnt)
        assert xp.send_splits == [int(cnt[d * El:(d + 1) * El].sum()) for d in range(world)]
        assert xp.recv_splits == [int(allc[s][rank * El:(rank + 1) * El].sum()) for s in range(world)]
        own = torch.empty(xp.n_recv, H, dtype=torch.float64)
        ex.to_owners(src, xp, own)
        expect = []
        for e in range(rank * El, (rank + 1) * El):
            for s in range(world):
                for i in range(int(allc[s][e])):
                    expect.append([s * 1e6 + e * 1e3 + i + c * 1e-3 for c in range(H)])
        assert torch.equal(own, torch.tensor(expect, dtype=torch.float64).reshape(-1, H))
        back = torch.empty_like(src)
        ex.to_sources(own * 2, xp, back)
        assert torch.equal(back, src * 2)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world,E,empty_rank", [(2, 8, -1), (3, 12, -1), (4, 16, -1), (2, 8, 1)])
def test_exchange_roundtrip_gloo(world, E, empty_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, E, 3, q, empty_rank)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res
