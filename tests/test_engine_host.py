"""Host-side argument checks of the engine (no GPU): tensors whose sizes do
not match the declared shapes are refused before any kernel could read past
them, and CPU tensors never reach a kernel (there is no CPU fallback)."""
import pytest
import torch

from usaf_b200 import engine
from usaf_b200.engine import Projection, _check_act


def _q4(E, R, C, gs=128):
    n = E * R * C
    return (torch.zeros(n // gs, gs // 2, dtype=torch.int8),
            torch.ones(n // gs, dtype=torch.float16), torch.zeros(n // gs, dtype=torch.float16))


def test_check_act():
    t = torch.zeros(4, 8, dtype=torch.bfloat16)
    _check_act("x", t, (4, 8), torch.bfloat16)
    with pytest.raises(ValueError):
        _check_act("x", t, (8, 4), torch.bfloat16)
    with pytest.raises(TypeError):
        _check_act("x", t, (4, 8), torch.float32)
    with pytest.raises(ValueError):
        _check_act("x", t.t(), (8, 4), torch.bfloat16)


@pytest.mark.parametrize("bad", ["q", "s", "z", "q_dtype", "s_dtype"])
def test_projection_rejects_mismatched_int4_tensors(bad):
    q, s, z = _q4(2, 16, 256)
    if bad == "q":
        q = q[:-1]
    elif bad == "s":
        s = s[:-1]
    elif bad == "z":
        z = torch.zeros(z.numel() + 1, dtype=torch.float16)
    elif bad == "q_dtype":
        q = q.to(torch.int32)
    else:
        s = s.float()
    with pytest.raises(ValueError):
        Projection(q, s, z, (2, 16, 256), 128, torch.float32)


def test_projection_rejects_straddling_groups():
    q, s, z = _q4(1, 3, 128)
    with pytest.raises(ValueError):
        Projection(q, s, z, (1, 2, 192), 128, torch.float32)


def test_projection_bf16_needs_a_device():
    q, s, z = _q4(2, 16, 256)
    with pytest.raises(TypeError):        # tensor-core copies are built on the device
        Projection(q, s, z, (2, 16, 256), 128, torch.bfloat16)


def test_overlay_checks_before_any_kernel():
    q, s, z = _q4(2, 16, 256)
    p = Projection(q, s, z, (2, 16, 256), 128, torch.float32)   # fp32: no device copies
    with pytest.raises(ValueError):       # index past the tensor
        p.set_overlay(torch.tensor([0, p.numel()]), torch.zeros(2))
    with pytest.raises(ValueError):       # negative index
        p.set_overlay(torch.tensor([-1, 3]), torch.zeros(2))
    with pytest.raises(ValueError):       # one master per coordinate
        p.set_overlay(torch.tensor([1, 3]), torch.zeros(3))
    with pytest.raises(TypeError):        # valid arguments, CPU tensors: no fallback
        p.set_overlay(torch.tensor([1, 3]), torch.zeros(2))
    assert p.n_ov == 0                    # a refused overlay leaves the projection as it was


def test_block_workspace_needs_a_device():
    dims = engine.BlockDims(T=8, H=256, E=4, I=128, top_k=2, norm_topk_prob=True,
                            dtype=torch.bfloat16)
    with pytest.raises(TypeError):
        engine.MoEBlock(dims, "cpu")
