"""The allocation-free split-K GEMM entry point, laya_b200_gemm_splitk_noalloc.

It exists for callers that cannot allocate device memory (a serving stack whose caching allocator
reserves the GPU's memory up front, a plugin host that forbids allocation in its callbacks): its
scratch is a fixed array in the library's device image instead of a cudaMalloc'd workspace. These
checks call it through the C ABI twice in a row, on two different problems, and compare each result
with the allocating entry point laya_b200_gemm_splitk and with an fp64 reference, at the tolerances
of the other GEMM tests (1e-4 relative for fp32 results, 1e-2 for bf16). The second call inherits the
array from the first (partials and error word), so it also checks that nothing a call leaves there
leaks into the next one. This file
sorts last so that a run stopping at its first failure has already run every other test.
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")

from layamd_b200 import load_lib

pytestmark = pytest.mark.gpu

EPI_STORE, EPI_RESID = 0, 3
OUT_BF16, OUT_F32 = 0, 2


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def _call(fn, A, W, out, M, N, K, splits, epi=EPI_STORE, out_mode=OUT_F32, resid=None, bias=None):
    return fn(_p(A), _p(W), _p(out), _p(resid), _p(bias), M, N, K, 1, epi, out_mode, 0, 128,
              None, None, None, 0, 0, splits, None, 1)


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    torch.cuda.set_device(0)
    return load_lib()


def test_noalloc_matches_allocating_entry_two_calls_in_a_row(lib):
    g = torch.Generator(device="cuda").manual_seed(7)
    # call 1: MLP-out shape, fp32 residual add with bias, K split in 4 slices
    M1, N1, K1 = 512, 1024, 2624
    A1 = torch.randn(M1, K1, device="cuda", generator=g).bfloat16()
    W1 = (0.02 * torch.randn(N1, K1, device="cuda", generator=g)).bfloat16()
    b1 = torch.randn(N1, device="cuda", generator=g)
    x0 = torch.randn(M1, N1, device="cuda", generator=g)
    # call 2: QKV-like shape with ragged rows, bf16 store, K split in 3 slices
    M2, N2, K2 = 300, 3072, 1024
    A2 = torch.randn(M2, K2, device="cuda", generator=g).bfloat16()
    W2 = (0.02 * torch.randn(N2, K2, device="cuda", generator=g)).bfloat16()

    x_na = x0.clone()
    o_na = torch.zeros(M2, N2, device="cuda", dtype=torch.bfloat16)
    na = lib.laya_b200_gemm_splitk_noalloc
    assert _call(na, A1, W1, None, M1, N1, K1, 4, epi=EPI_RESID, resid=x_na, bias=b1) == 0
    assert _call(na, A2, W2, o_na, M2, N2, K2, 3, out_mode=OUT_BF16) == 0

    x_al = x0.clone()
    o_al = torch.zeros(M2, N2, device="cuda", dtype=torch.bfloat16)
    al = lib.laya_b200_gemm_splitk
    assert _call(al, A1, W1, None, M1, N1, K1, 4, epi=EPI_RESID, resid=x_al, bias=b1) == 0
    assert _call(al, A2, W2, o_al, M2, N2, K2, 3, out_mode=OUT_BF16) == 0
    torch.cuda.synchronize()

    ref1 = x0.double() + A1.double() @ W1.double().T + b1.double()
    ref2 = A2.double() @ W2.double().T
    assert _rel(x_na, x_al) < 1e-4 and _rel(x_na, ref1) < 1e-4
    assert _rel(o_na, o_al) < 1e-2 and _rel(o_na, ref2) < 1e-2


def test_noalloc_rejects_problems_beyond_its_scratch(lib):
    # 4096 x 5248 in 8 slices needs 172 M partial floats, far beyond the 4 Mi the array holds
    M, N, K = 4096, 5248, 1024
    A = torch.zeros(M, K, device="cuda", dtype=torch.bfloat16)
    W = torch.zeros(N, K, device="cuda", dtype=torch.bfloat16)
    out = torch.full((M, N), 3.0, device="cuda")
    assert _call(lib.laya_b200_gemm_splitk_noalloc, A, W, out, M, N, K, 8) == -7
    torch.cuda.synchronize()
    assert bool((out == 3.0).all())  # nothing was launched
