"""SparseAdam keeps its state on the parameters' CUDA device: CPU
parameters are refused at construction (no CPU fallback)."""
import pytest
import torch

from usaf_b200.sparse_optim import SparseAdam


def test_cpu_parameters_refused():
    params = {"w": torch.nn.Parameter(torch.ones(10))}
    with pytest.raises(TypeError):
        SparseAdam(params, active_idx={"w": torch.tensor([0, 1])})


def test_empty_selection_builds_no_state():
    # a tensor with no active coordinates is skipped before any device is touched
    params = {"w": torch.nn.Parameter(torch.ones(10))}
    opt = SparseAdam(params, active_idx={"w": torch.zeros(0, dtype=torch.long)})
    assert opt.num_active_params == 0
    assert opt.state_dict()["step"] == 0
