"""Reference regrouping of expert-parallel rows, for the tests: received rows
are in (source rank, local expert) block order; the owner wants
(local expert, source rank).  Pure torch index arithmetic on any device."""
import torch


def regroup_index(counts: torch.Tensor) -> torch.Tensor:
    """dst[i] = expert-major position of received row i; counts [W, El]."""
    W, El = counts.shape
    c = counts.to(torch.int64).cpu()
    src_start = torch.zeros(W * El + 1, dtype=torch.int64)
    src_start[1:] = torch.cumsum(c.reshape(-1), 0)
    dst_start = torch.zeros(W, El, dtype=torch.int64)
    run = 0
    for e in range(El):
        for s in range(W):
            dst_start[s, e] = run
            run += int(c[s, e])
    n = int(src_start[-1])
    dst = torch.empty(n, dtype=torch.int64)
    for s in range(W):
        for e in range(El):
            b = s * El + e
            a0, a1 = int(src_start[b]), int(src_start[b + 1])
            dst[a0:a1] = dst_start[s, e] + torch.arange(a1 - a0)
    return dst


def permute(counts, rows_in, rows_out, inverse, err=None):
    dst = regroup_index(counts).to(rows_in.device)
    if inverse:
        rows_out.copy_(rows_in[dst])
    else:
        rows_out[dst] = rows_in
