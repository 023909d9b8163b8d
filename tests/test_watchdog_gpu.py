"""The device watchdog on a B200: every pipeline wait of the GEMM and attention kernels is bounded,
and a wait that runs out records an error code and lets its kernel end instead of hanging the GPU
(the reference engine has no such path; it exits on any GPU error). The self-test entry point
``laya_b200_watchdog_selftest`` makes one thread wait on a barrier phase that nothing completes; no
fault, trap or endless loop is involved. The recorded code is then read back through
``laya_b200_kernel_error``, the route for errors of asynchronous calls, and the same process runs an
ordinary GEMM through the C ABI, showing that the context is still usable."""
import ctypes

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from layamd_b200 import LIB_PATH  # noqa: E402

ERR_SELF_TEST = 30
BUDGET_CYCLES = 1 << 31


def test_wait_runs_out_and_context_stays_usable():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    L = ctypes.CDLL(LIB_PATH)
    i, vp = ctypes.c_int, ctypes.c_void_p
    L.laya_b200_watchdog_selftest.restype = i
    L.laya_b200_watchdog_selftest.argtypes = [i, ctypes.POINTER(i), ctypes.POINTER(ctypes.c_longlong),
                                              ctypes.POINTER(ctypes.c_float)]
    code, cycles, ms = i(-1), ctypes.c_longlong(0), ctypes.c_float(0)
    assert L.laya_b200_watchdog_selftest(0, ctypes.byref(code), ctypes.byref(cycles), ctypes.byref(ms)) == 0
    print("watchdog self-test: code %d after %d SM cycles, %.1f ms" % (code.value, cycles.value, ms.value))
    assert code.value == ERR_SELF_TEST
    # the wait gave up on its budget (it never saw the phase complete), within a few SM-clock seconds
    assert BUDGET_CYCLES < cycles.value < BUDGET_CYCLES + (1 << 28)
    assert 0.3e3 < ms.value < 10e3

    # The code stays in the error word of the kernel-level entry points until it is read, so a kernel
    # of an asynchronous (sync = 0) entry call that ran out of its wait cannot go unreported: the
    # self-test refuses to run over it, an asynchronous GEMM leaves it alone, and the getter reads
    # and clears it.
    L.laya_b200_kernel_error.restype = i
    L.laya_b200_kernel_error.argtypes = [i]
    assert L.laya_b200_watchdog_selftest(0, ctypes.byref(code), ctypes.byref(cycles), ctypes.byref(ms)) == -3

    # the context is intact: an ordinary GEMM through the C ABI right after
    L.laya_b200_gemm.restype = i
    L.laya_b200_gemm.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, i, i, i, i, vp, vp, vp, i, i, vp, i]
    g = torch.Generator(device="cuda").manual_seed(30)
    M, N, K = 256, 512, 1024
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.02 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    out = torch.full((M, N), float("nan"), device="cuda")
    torch.cuda.synchronize()

    def gemm(sync):
        return L.laya_b200_gemm(ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(W.data_ptr()),
                                ctypes.c_void_p(out.data_ptr()), None, None, M, N, K, 1, 0, 2, 0, 128, None, None,
                                None, 0, 0, None, sync)

    assert gemm(0) == 0  # asynchronous: cannot report, must not clear
    assert L.laya_b200_kernel_error(0) == ERR_SELF_TEST
    assert L.laya_b200_kernel_error(0) == 0  # read and cleared
    assert gemm(1) == 0
    ref = A.double() @ W.double().T
    assert float((out.double() - ref).abs().max() / ref.abs().max()) < 1e-4
