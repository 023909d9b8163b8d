"""Fine-tune export check (layamd_b200.export) on CPU: the reference's own verdicts and messages on the
golden cases (tests/golden/make_export_golden.py), the restored base files, and this engine's own
model-shape limits."""
import filecmp
import json
import os
import shutil

import pytest

from layamd_b200 import export as X
from tests import export_cases

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLD, "export_golden.json")) as f:
        return json.load(f)


@pytest.mark.parametrize("name", export_cases.CASES)
def test_verdicts_match_reference(tmp_path, capsys, golden, name):
    base = export_cases.base_checkpoint()
    out = export_cases.build(base, str(tmp_path), name)
    rc = X.main([base, out])
    lines = capsys.readouterr().out.rstrip("\n").split("\n")
    want = golden[name]
    assert rc == want["rc"]
    assert lines[0] == want["lines"][0]
    assert sorted(lines[1:]) == sorted(want["lines"][1:])  # the reference lists shape errors in set order
    # the trainer's re-saved files are replaced by the base's, its resume copy removed
    assert filecmp.cmp(os.path.join(base, "encoder", "config.json"), os.path.join(out, "encoder", "config.json"),
                       shallow=False)
    assert filecmp.cmp(os.path.join(base, "tokenizer", "tokenizer.json"),
                       os.path.join(out, "tokenizer", "tokenizer.json"), shallow=False)
    assert not os.path.exists(os.path.join(out, "checkpoint_latest"))


def test_engine_shape_limits(tmp_path):
    """A base whose shape this engine's kernels do not take is refused with the reason."""
    base0 = export_cases.base_checkpoint()
    base = str(tmp_path / "base")
    shutil.copytree(base0, base)
    with open(os.path.join(base, "encoder", "config.json")) as f:
        enc = json.load(f)
    enc.update(num_attention_heads=4, intermediate_size=200)  # head_dim 32, GeGLU width not a multiple of 64
    with open(os.path.join(base, "encoder", "config.json"), "w") as f:
        json.dump(enc, f)
    out = export_cases.build(base, str(tmp_path), "fp16")
    errs = X.check(base, out)
    assert "head_dim 32.0: the attention kernels take 64" in errs
    assert "intermediate_size 200: the engine takes a multiple of 64" in errs


def test_usage(capsys):
    assert X.main([]) == 2
    assert "BASE_DIR OUT_DIR" in capsys.readouterr().out
