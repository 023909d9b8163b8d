"""Generates tests/golden/export_golden.json from the reference's own fine-tune export check
(test infrastructure).

Run in the build container, where the reference checkout is available (LAYA_REFERENCE):

    python tests/golden/make_export_golden.py

For every case of tests/export_cases.py (trainer output directories made from the tiny base
checkpoint) it runs the reference's finetune/export.py ``main(base, out)`` and records its exit code
and printed lines. tests/test_export_cpu.py runs layamd_b200.export on the same cases and compares.
"""
import contextlib
import importlib.util
import io
import json
import os
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from tests import export_cases  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
from oracle.ref_tools import reference_root  # noqa: E402

REF = reference_root()


def main():
    spec = importlib.util.spec_from_file_location("ref_export", os.path.join(REF, "finetune", "export.py"))
    ref = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(ref)
    base = export_cases.base_checkpoint()
    res = {}
    with tempfile.TemporaryDirectory() as root:
        for name in export_cases.CASES:
            out = export_cases.build(base, root, name)
            buf = io.StringIO()
            rc = 0
            with contextlib.redirect_stdout(buf):
                try:
                    ref.main(base, out)
                except SystemExit as e:
                    rc = int(e.code or 0)
            res[name] = {"rc": rc, "lines": buf.getvalue().rstrip("\n").split("\n")}
    with open(os.path.join(HERE, "export_golden.json"), "w") as f:
        json.dump(res, f, indent=1)
    print("wrote %d cases" % len(res))


if __name__ == "__main__":
    main()
