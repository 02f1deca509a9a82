"""SparseAdam on the device: the reference's own optimizer tests
(tests/test_sparse_optim.py:7-79 of the reference) on CUDA parameters, and
three steps of both parameter modes against the oracle's restatement of
usaf/sparse_optim.py:86-134 (rel <= 1e-6, fp32 state)."""
import pytest
import torch

from oracle import moe as omoe

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import usaf_b200  # noqa: F401
    return torch.device("cuda:0")


def test_init_with_idx(dev):
    from usaf_b200.sparse_optim import SparseAdam
    params = {"layer1.weight": torch.nn.Parameter(torch.randn(10, 10, device=dev)),
              "layer2.weight": torch.nn.Parameter(torch.randn(5, 5, device=dev))}
    active = {"layer1.weight": torch.tensor([0, 1, 2, 3, 4]), "layer2.weight": torch.tensor([0, 5, 10])}
    opt = SparseAdam(params, active_idx=active, lr=1e-3)
    assert opt.num_active_params == 8
    assert opt.optimizer_memory_mb > 0


def test_step_touches_only_active(dev):
    from usaf_b200.sparse_optim import SparseAdam
    param = torch.nn.Parameter(torch.ones(10, device=dev))
    opt = SparseAdam({"w": param}, active_idx={"w": torch.tensor([0, 1, 2, 3, 4])}, lr=1.0)
    param[:5].sum().backward()
    opt.step()
    assert param[0].item() < 1.0
    assert param[5].item() == 1.0


def test_step_without_grad_is_a_no_op(dev):
    from usaf_b200.sparse_optim import SparseAdam
    param = torch.nn.Parameter(torch.ones(10, device=dev))
    opt = SparseAdam({"w": param}, active_idx={"w": torch.tensor([0, 1])}, lr=1.0)
    opt.step()
    assert torch.equal(param.detach(), torch.ones(10, device=dev))


def test_compact_grads(dev):
    from usaf_b200.sparse_optim import SparseAdam
    param = torch.nn.Parameter(torch.ones(10, device=dev))
    opt = SparseAdam({"w": param}, active_idx={"w": torch.tensor([0, 1, 2])}, lr=1.0)
    opt.step(compact_grads={"w": torch.ones(3, device=dev)})
    assert param[0].item() < 1.0
    assert param[3].item() == 1.0


def test_zero_grad_and_state_dict(dev):
    from usaf_b200.sparse_optim import SparseAdam
    param = torch.nn.Parameter(torch.randn(10, device=dev))
    opt = SparseAdam({"w": param}, active_idx={"w": torch.tensor([0, 1])})
    param.grad = torch.ones(10, device=dev)
    opt.zero_grad()
    assert torch.count_nonzero(param.grad) == 0
    sd = opt.state_dict()
    assert set(sd) >= {"step", "m", "v"} and sd["step"] == 0
    assert not sd["m"]["w"].is_cuda          # checkpoint-compatible CPU tensors
    sd["step"] = 5
    opt.load_state_dict(sd)
    assert opt._step == 5


@pytest.mark.parametrize("compact", [True, False])
def test_three_steps_vs_oracle(dev, compact):
    from usaf_b200.sparse_optim import SparseAdam
    g = torch.Generator().manual_seed(3)
    n_full, n_act = 4096, 700
    idx = torch.randperm(n_full, generator=g)[:n_act]
    if compact:
        p0 = torch.randn(n_act, generator=g)
    else:
        p0 = torch.randn(n_full, generator=g)
    grads = [torch.randn(n_act if compact else n_full, generator=g) for _ in range(3)]
    ref_p = p0.clone()
    ref = omoe.SparseAdam({"w": ref_p}, {"w": idx}, lr=1e-2, weight_decay=0.01, compact_params=compact)
    dev_p = torch.nn.Parameter(p0.clone().to(dev), requires_grad=False)
    opt = SparseAdam({"w": dev_p}, active_idx={"w": idx}, lr=1e-2, weight_decay=0.01,
                     compact_params=compact)
    for gr in grads:
        ref.step({"w": gr})
        if compact:
            opt.step(compact_grads={"w": gr.to(dev)})
        else:
            dev_p.grad = gr.to(dev)
            opt.step()
    got = dev_p.detach().cpu()
    rel = ((got.double() - ref_p.double()).norm() / ref_p.double().norm()).item()
    assert rel <= 1e-6, rel
    if not compact:   # inactive coordinates untouched
        mask = torch.ones(n_full, dtype=torch.bool)
        mask[idx] = False
        assert torch.equal(got[mask], p0[mask])
