"""The `usaf train` surface (usaf_b200/train.py) against the reference's own
CLI, on the CPU: tests/golden/make_golden.py ran the reference's parse_args
(usaf/train.py:131-171) on several command lines and its dataset loader
(:173-194) on a seeded JSONL; the configurations and the train / eval /
held-out splits must be identical here.  The device path refuses --no-cuda."""
import dataclasses
import json
import os
import sys

import pytest

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden"))


def _fixture(golden_dir):
    with open(os.path.join(golden_dir, "cli.json")) as f:
        return json.load(f)


def test_parse_args_matches_reference(golden_dir):
    from usaf_b200 import train
    fx = _fixture(golden_dir)
    for args, cfg in zip(fx["args"], fx["configs"]):
        got = dataclasses.asdict(train.parse_args(args))
        if "--cuda" not in args and "--no-cuda" not in args:
            # the default follows torch.cuda.is_available() on the host that parses
            got["use_cuda"] = cfg["use_cuda"]
        assert got == cfg, args


def test_dataset_split_matches_reference(golden_dir, tmp_path):
    from make_golden import cli_dataset_lines
    from usaf_b200 import train
    fx = _fixture(golden_dir)
    path = tmp_path / "data.jsonl"
    path.write_text("\n".join(cli_dataset_lines()) + "\n")
    tr, ev, he = train.load_dataset(str(path), 8)
    assert [s["id"] for s in tr] == fx["dataset"]["train"]
    assert [s["id"] for s in ev] == fx["dataset"]["eval"]
    assert [s["id"] for s in he] == fx["dataset"]["heldout"]


def test_no_cuda_is_refused(tmp_path):
    from usaf_b200 import train
    with pytest.raises(SystemExit, match="no CPU path"):
        train.main(["--model", str(tmp_path), "--dataset", str(tmp_path / "d.jsonl"), "--no-cuda"])
