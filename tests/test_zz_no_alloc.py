"""The allocation-free split-K GEMM entry point, laya_b200_gemm_splitk_noalloc.

It exists for callers that cannot allocate device memory (a serving stack whose caching allocator
reserves the GPU's memory up front, a plugin host that forbids allocation in its callbacks): its
scratch is a fixed array in the library's device image instead of a cudaMalloc'd workspace. These
checks call it through the C ABI twice in a row, on two different problems, and compare each result
with the allocating entry point laya_b200_gemm_splitk and with an fp64 reference, at the tolerances
of the other GEMM tests (1e-4 relative for fp32 results, 1e-2 for bf16). The second call inherits the
array from the first (partials and error word), so it also checks that nothing a call leaves there
leaks into the next one. A further check reads the device's free memory around a call to show that
it allocates nothing. This file sorts last so that a run stopping at its first failure has already
run every other test.
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


def test_noalloc_call_allocates_no_device_memory(lib):
    """The property the entry point exists for. After a warm-up call (set-up, and the lazy loading of
    the kernels it launches), a call on another shape leaves the device's free memory unchanged,
    while the allocating entry point grows its workspace for a problem larger than any before it."""
    g = torch.Generator(device="cuda").manual_seed(11)
    shapes = [(384, 1024, 2624, 4), (256, 2048, 1024, 2)]  # splits x M x N <= 4 Mi partials
    ins = []
    for M, N, K, sp in shapes:
        A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
        W = (0.02 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
        ins.append((A, W, torch.zeros(M, N, device="cuda"), M, N, K, sp))
    Mb, Nb, Kb, spb = 4096, 3072, 1024, 8  # 100 M partials (400 MB), beyond every other test's workspace
    Ab = torch.randn(Mb, Kb, device="cuda", generator=g).bfloat16()
    Wb = (0.02 * torch.randn(Nb, Kb, device="cuda", generator=g)).bfloat16()
    ob = torch.zeros(Mb, Nb, device="cuda")
    na = lib.laya_b200_gemm_splitk_noalloc
    A, W, o, M, N, K, sp = ins[0]
    assert _call(na, A, W, o, M, N, K, sp) == 0  # warm-up
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    A, W, o, M, N, K, sp = ins[1]
    assert _call(na, A, W, o, M, N, K, sp) == 0
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, "the allocation-free entry changed free device memory by %d bytes" % (free0 - free1)
    assert _rel(o, A.double() @ W.double().T) < 1e-4
    assert _call(lib.laya_b200_gemm_splitk, Ab, Wb, ob, Mb, Nb, Kb, spb) == 0
    torch.cuda.synchronize()
    free2 = torch.cuda.mem_get_info()[0]
    # the allocating entry did grow its workspace: it frees its previous, smaller one (a few tens of
    # MB from the earlier tests at most) and allocates 400 MB
    assert free1 - free2 >= 0.75 * spb * Mb * Nb * 4


def test_split_count_beyond_the_k_blocks_is_rejected(lib):
    """Every K slice must own a K block, or its partial plane would hold an accumulator nobody wrote:
    K = 128 has two 64-wide blocks, so 4 slices are refused by both split-K entries before anything
    is launched, and 2 slices give the right product."""
    g = torch.Generator(device="cuda").manual_seed(12)
    M, N, K = 256, 512, 128
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.02 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    for fn in (lib.laya_b200_gemm_splitk_noalloc, lib.laya_b200_gemm_splitk):
        out = torch.full((M, N), 3.0, device="cuda")
        assert _call(fn, A, W, out, M, N, K, 4) == -2
        torch.cuda.synchronize()
        assert bool((out == 3.0).all())
        assert _call(fn, A, W, out, M, N, K, 2) == 0
        torch.cuda.synchronize()
        assert _rel(out, A.double() @ W.double().T) < 1e-4
    assert lib.laya_b200_kernel_error(0) == 0  # and no kernel recorded an error


def test_noalloc_rejects_problems_beyond_its_scratch(lib):
    # 4096 x 5248 in 8 slices needs 172 M partial floats, far beyond the 4 Mi the array holds
    M, N, K = 4096, 5248, 1024
    A = torch.zeros(M, K, device="cuda", dtype=torch.bfloat16)
    W = torch.zeros(N, K, device="cuda", dtype=torch.bfloat16)
    out = torch.full((M, N), 3.0, device="cuda")
    assert _call(lib.laya_b200_gemm_splitk_noalloc, A, W, out, M, N, K, 8) == -7
    torch.cuda.synchronize()
    assert bool((out == 3.0).all())  # nothing was launched
