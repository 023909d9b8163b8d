"""The benchmark's roofline arithmetic, restated by hand (CPU only): the algorithmic FLOPs of the
encoder GEMM classes and the algorithmic bytes per launch of the HBM-bound stages that bench.py
divides by device time, and the split between the tensor-bound GEMMs and the attention
out-projection."""
import importlib.util
import os
import sys

import pytest

from layamd_b200.synthetic import synth, workloads

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    argv = sys.argv
    sys.argv = ["bench.py"]
    try:
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    return mod


def test_encoder_gemm_flops_are_2mnk(bench):
    arch = synth.ARCHS["large"]
    qs = workloads.c2(arch, seed=1)
    T = sum(len(q["ids"]) for q in qs)
    assert T == 52287
    fl = bench.encoder_gemm_flops(qs, arch)
    D, I, NL = 1024, 2624, 28
    assert fl["gemm_qkv"] == 2.0 * T * D * 3 * D * NL
    assert fl["gemm_attn_out"] == 2.0 * T * D * D * NL
    assert fl["gemm_mlp_in"] == 2.0 * T * D * 2 * I * NL
    assert fl["gemm_mlp_out"] == 2.0 * T * I * D * NL


def test_hbm_bytes_per_launch(bench):
    arch = synth.ARCHS["large"]
    qs = workloads.c2(arch, seed=1)
    T, D = 52287, 1024
    prof = {"attn_global": (2.4, 10), "attn_sliding": (2.7, 18), "ln": (3.2, 56), "embed_ln": (0.09, 1),
            "gemm_attn_out": (3.5, 28)}
    out = bench.hbm_rooflines(qs, arch, prof)
    # attention: q, k, v read once (6D bf16 bytes) and the output row written (2D)
    assert out["attn_global"]["bytes_per_launch"] == 8 * D * T
    assert out["attn_sliding"]["bytes_per_launch"] == 8 * D * T
    # LayerNorm: fp32 x in (4D), bf16 out (2D); the encoder's last one also writes x back (+4D once)
    assert out["ln"]["bytes_per_launch"] == (56 * 6 * D * T + 4 * D * T) // 56
    # out-projection: bf16 rows in (2D), fp32 residual read and written (8D), the D x D weight once
    assert out["gemm_attn_out"]["bytes_per_launch"] == 10 * D * T + 2 * D * D
    for k in ("attn_global", "attn_sliding", "ln", "embed_ln", "gemm_attn_out"):
        ms, n = prof[k]
        byt = out[k]["bytes_per_launch"] * n
        assert abs(out[k]["achieved_gbs"] - byt / (ms / 1e3) / 1e9) < 0.1
        assert abs(out[k]["frac"] - out[k]["achieved_gbs"] / out["peak_gbs"]) < 1e-3


def test_out_projection_is_balanced_between_its_two_bounds(bench):
    """Why the out-projection is reported with the HBM-bound stages: at the C2 shape its FLOPs at the
    sustained tensor peak and its bytes at the copy bandwidth take about as long."""
    T, D = 52287, 1024
    flop_s = 2.0 * T * D * D / 1331.0e12
    byte_s = (10 * D * T + 2 * D * D) / 6549.1e9
    assert 0.8 < flop_s / byte_s < 1.25
    # the MLP-out projection (K = I) is clearly tensor-bound
    I = 2624
    flop_s = 2.0 * T * I * D / 1331.0e12
    byte_s = (2 * I * T + 8 * D * T + 2 * D * I) / 6549.1e9
    assert flop_s / byte_s > 1.5
