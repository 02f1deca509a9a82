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


def test_pair_capacity():
    assert engine.pair_capacity(4096, 128, 8) == 4096 * 16           # default: room for 2 x top_k
    assert engine.pair_capacity(8192, 128, 8, 1.25) == 8192 * 10
    assert engine.pair_capacity(64, 8, 2) == 64 * 4
    assert engine.pair_capacity(64, 3, 2) == 64 * 3                  # never more than E per token
    with pytest.raises(ValueError):
        engine.pair_capacity(64, 8, 2, 0.5)


def test_workspace_policy():
    from usaf_b200 import qwen3moe
    try:
        qwen3moe.configure_workspaces(pair_factor=1.25, share_backward=True)
        assert qwen3moe._POLICY == {"pair_factor": 1.25, "share_backward": True}
        with pytest.raises(ValueError):
            qwen3moe.configure_workspaces(pair_factor=0.9)
    finally:
        qwen3moe.configure_workspaces()
    assert qwen3moe._POLICY == {"pair_factor": 2.0, "share_backward": False}


def test_model_built_without_dense_experts():
    """The C3 setup builds its experts without dense tensors (their weights
    come from the int4 store); everything else is built as usual, and the
    class is restored afterwards."""
    from transformers.models.qwen3_moe.configuration_qwen3_moe import Qwen3MoeConfig
    from transformers.models.qwen3_moe.modeling_qwen3_moe import Qwen3MoeForCausalLM
    from usaf_b200 import qwen3moe
    cfg = Qwen3MoeConfig(vocab_size=64, hidden_size=32, intermediate_size=64, num_hidden_layers=2,
                         num_attention_heads=4, num_key_value_heads=2, head_dim=8,
                         moe_intermediate_size=16, num_experts=4, num_experts_per_tok=2,
                         norm_topk_prob=True)
    with torch.device("cpu"), qwen3moe.without_dense_experts():
        lean = Qwen3MoeForCausalLM(cfg)
    for layer in lean.model.layers:
        assert layer.mlp.experts.gate_up_proj.numel() == 0
        assert layer.mlp.experts.down_proj.numel() == 0
        assert layer.mlp.gate.weight.shape == (4, 32) and layer.mlp.gate.weight.abs().sum() > 0
        assert not layer.mlp.experts.gate_up_proj.is_meta
    full = Qwen3MoeForCausalLM(cfg)
    assert full.model.layers[0].mlp.experts.gate_up_proj.shape == (4, 32, 32)


def test_shared_scratch_must_match_the_block():
    dims = engine.BlockDims(T=8, H=256, E=4, I=128, top_k=2, norm_topk_prob=True,
                            dtype=torch.bfloat16)
    P_cap = engine.pair_capacity(8, 4, 2, 2)
    wrong = engine.BackwardScratch(P_cap + 1, 8, 256, 4, 128, torch.bfloat16, "cpu")
    with pytest.raises(ValueError):
        engine.MoEBlock(dims, "cpu", 2, wrong)
    right = engine.BackwardScratch(P_cap, 8, 256, 4, 128, torch.bfloat16, "cpu")
    assert right.dcur.shape == (P_cap, 256) and right.dgu.shape == (P_cap, 256)
    with pytest.raises(TypeError):        # sizes agree; CPU tensors never reach a kernel
        engine.MoEBlock(dims, "cpu", 2, right)


def test_rigl_merge_with_an_empty_active_set():
    """The grown budget is len(old) - len(kept): an empty old set stays empty
    (and never reaches the device search)."""
    from usaf_b200 import rigl
    empty = torch.empty(0, dtype=torch.long)
    fin, vals = rigl.merge(empty, torch.tensor([3, 1, 2]), torch.empty(0), torch.zeros(8))
    assert fin.numel() == 0 and vals.numel() == 0
    fin, vals = rigl.merge(torch.tensor([4, 2]), None, torch.tensor([0.5, 0.25]), torch.zeros(8))
    assert fin.tolist() == [4, 2] and vals.tolist() == [0.5, 0.25]


def test_csr_order_refuses_out_of_range_indices():
    q, s, z = _q4(2, 16, 256)
    p = Projection(q, s, z, (2, 16, 256), 128, torch.float32)
    with pytest.raises(IndexError):
        p.csr_order(torch.tensor([5, p.numel()]))
    with pytest.raises(IndexError):
        p.csr_order(torch.tensor([-3]))


def test_dequantize_checks_the_layout_sizes():
    from usaf_b200.quantization import dequantize_4bit
    q, s, z = _q4(1, 4, 256)                        # 1024 elements: 8 groups of 128
    with pytest.raises(ValueError):
        dequantize_4bit(q[:-1], s, z, (4, 256))
    with pytest.raises(ValueError):
        dequantize_4bit(q, s[:-1], z, (4, 256))
    with pytest.raises(ValueError):
        dequantize_4bit(q, s, z.float(), (4, 256))
    with pytest.raises(ValueError):
        dequantize_4bit(q, s, z, (8, 256))          # shape larger than the codes
    with pytest.raises(TypeError):                  # consistent sizes, CPU tensors: no fallback
        dequantize_4bit(q, s, z, (4, 256))
