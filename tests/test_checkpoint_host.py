"""usaf_b200.checkpoint save / load / metadata on the host (the reference's own
checkpoint tests, tests/test_checkpoint.py:13-88, with the same inputs)."""
import os
import tempfile

import pytest
import torch


def test_save_load_roundtrip():
    from usaf_b200.checkpoint import load_sparse_checkpoint, save_sparse_checkpoint
    masters = {"w1": torch.nn.Parameter(torch.tensor([1.0, 2.0, 3.0])),
               "w2": torch.nn.Parameter(torch.tensor([4.0, 5.0]))}
    active_idx = {"w1": torch.tensor([0, 10, 20], dtype=torch.long),
                  "w2": torch.tensor([5, 15], dtype=torch.long)}
    opt_state = {"step": 3, "m": {"w1": torch.zeros(3)}, "v": {"w1": torch.zeros(3)}}
    config = {"model": "test-model", "steps": 100, "frac": 0.005, "lr": 2e-4}
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "ckpt.pt")
        save_sparse_checkpoint(path, masters, active_idx, opt_state, config, step=5,
                               losses=[2.5, 2.3, 2.1], train_layers=[11, 12, 13], metric=2.1)
        loaded = load_sparse_checkpoint(path)
        assert loaded["format"] == "usaf-sparse-v1"
        assert loaded["step"] == 5 and len(loaded["losses"]) == 3 and loaded["metric"] == 2.1
        assert torch.equal(loaded["active_idx"]["w1"], active_idx["w1"])
        assert torch.equal(loaded["masters"]["w2"], masters["w2"].detach())
        assert loaded["config"]["model"] == "test-model"
        assert loaded["train_layers"] == [11, 12, 13]
        assert loaded["optimizer"]["step"] == 3


def test_metadata_and_overwrite():
    from usaf_b200.checkpoint import (get_checkpoint_metadata, load_sparse_checkpoint,
                                      save_sparse_checkpoint)
    masters = {"w": torch.nn.Parameter(torch.tensor([1.0, 2.0]))}
    active_idx = {"w": torch.tensor([0, 5], dtype=torch.long)}
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "ckpt.pt")
        save_sparse_checkpoint(path, masters, active_idx, {}, {"model": "test"}, step=10,
                               losses=[1.0], train_layers=[0])
        meta = get_checkpoint_metadata(path)
        assert meta["step"] == 10 and meta["n_active"] == 2 and meta["n_masters"] == 1
        assert meta["format"] == "usaf-sparse-v1"
        save_sparse_checkpoint(path, masters, active_idx, {}, {}, step=11, losses=[], train_layers=[0])
        assert load_sparse_checkpoint(path)["step"] == 11


def test_load_invalid_raises():
    from usaf_b200.checkpoint import load_sparse_checkpoint
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "bad.pt")
        torch.save({"format": "unknown"}, path)
        with pytest.raises(ValueError):
            load_sparse_checkpoint(path)
