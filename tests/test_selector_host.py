"""Host-side behaviour of the device selectors (no GPU needed): the reselect
counter of DynamicSelector (reference tests/test_selector.py:41-47) and the
refusal of CPU score tensors (there is no CPU fallback)."""
import pytest
import torch


def test_dynamic_selector_counter():
    from usaf_b200.selector import DynamicSelector
    sel = DynamicSelector(initial_k=100, reselect_every_n_steps=50, selection="topk")
    assert sel.should_reselect() is False
    for _ in range(48):
        sel.should_reselect()
    assert sel.should_reselect() is True
    assert sel.should_reselect() is False


def test_cpu_scores_rejected():
    from usaf_b200.selector import ThresholdSelector, TopKSelector
    with pytest.raises(TypeError):
        TopKSelector(3).select({"w": torch.tensor([1.0, 2.0])})
    with pytest.raises(TypeError):
        ThresholdSelector(50.0).select({"w": torch.tensor([1.0, 2.0])})
