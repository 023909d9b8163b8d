"""layamd_b200.golden_parity (the reference's test_parity.cpp check plus per-layer comparison) on a
golden set in the reference's layout: one written from the oracle for the tiny checkpoint, and the
reference's own set for a real checkpoint when LAYA_MODEL_DIR and LAYA_GOLDEN_DIR point to them."""
import io
import os

import pytest

torch = pytest.importorskip("torch")

from layamd_b200 import golden_parity as G  # noqa: E402
from layamd_b200.synthetic import synth  # noqa: E402
from tests import golden_format  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture(scope="module")
def tiny_golden(tmp_path_factory):
    ck = synth.checkpoint("tiny", 0)
    d = str(tmp_path_factory.mktemp("golden"))
    golden_format.write(ck, d)
    return ck, d


def test_fp32_parity_on_written_golden_set(tiny_golden):
    ck, d = tiny_golden
    res = G.run(ck, d, precision=1, out=io.StringIO())
    assert res["rows"] == 2 * 6 and res["fails"] == 0
    assert res["worst_prob"] <= 1e-4 and res["worst_layer"] <= 1e-3 and res["worst_api"] <= 2e-4
    assert set(res["layers"]["fill_ctx"]) >= {"emb", "enc0", "enc3", "final_norm", "head0", "head1"}


def test_bf16_on_written_golden_set(tiny_golden):
    ck, d = tiny_golden
    res = G.run(ck, d, precision=0, out=io.StringIO())
    assert res["fails"] == 0 and res["worst_prob"] < 0.01


@pytest.mark.skipif(not (os.environ.get("LAYA_MODEL_DIR") and os.environ.get("LAYA_GOLDEN_DIR")),
                    reason="real checkpoint and its golden set not available")
def test_reference_golden_set():
    res = G.run(os.environ["LAYA_MODEL_DIR"], os.environ["LAYA_GOLDEN_DIR"], precision=1)
    assert res["fails"] == 0
