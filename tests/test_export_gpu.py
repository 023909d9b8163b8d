"""A fine-tune export as the trainer writes it (fp16 matrices, bf16 LayerNorm gains) loads into the
engine and matches the oracle run on the same stored weights."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import model as om  # noqa: E402
from layamd_b200.synthetic import synth, workloads  # noqa: E402
from tests import export_cases  # noqa: E402
from tests.engine_helpers import Handle, act_rel, prob_delta  # noqa: E402

from layamd_b200 import export as X  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def test_fp16_export_serves_like_the_oracle(tmp_path):
    base = export_cases.base_checkpoint()
    out = export_cases.build(base, str(tmp_path), "fp16")
    assert X.main([base, out]) == 0
    o = om.Oracle(synth.load_weights(out), synth.load_arch(out))  # F16 / BF16 tensors read back as fp32
    qs = workloads.mixed(synth.ARCHS["tiny"], 24, seed=321, kmax=8)
    lo_o, ac_o, _ = o.forward_batch(qs)
    for precision, dp, da in ((1, 1e-4, 1e-3), (0, 0.01, 0.05)):
        h = Handle(out, precision)
        try:
            rc, lo, ac = h.forward(qs)
        finally:
            h.close()
        assert rc == 0
        assert prob_delta(lo, lo_o, qs) <= dp
        assert act_rel(ac, ac_o) <= da
    # the stored fp16 weights are not the base's fp32 ones: the check above is not vacuous
    w0, w1 = synth.load_weights(base), synth.load_weights(out)
    assert any(not np.array_equal(w0[k], w1[k]) for k in w0)
