"""Kernel parity of the tcgen05 GEMM (layamd_b200/csrc/gemm_tc.cu) through the C ABI entry point
``laya_b200_gemm``, against a plain PyTorch fp32/fp64 reference of the same op.

bn selects the tile: 128 / 256 (one CTA per 128 x bn tile) or 512 (CTA pair, 256 x 256, 2-SM MMA).
Tolerances (max|out-ref| / max|ref|): fp32-output bf16 GEMM 1e-4 (fp32 accumulation order only);
three-product split-bf16 (fp32-parity mode) 5e-5 against fp64 on the fp32 inputs; bf16 outputs 1e-2
(one bf16 rounding of the result).
"""
import ctypes
import math

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from layamd_b200 import LIB_PATH  # noqa: E402

EPI_STORE, EPI_ROPE, EPI_GEGLU, EPI_RESID = 0, 1, 2, 3
OUT_BF16, OUT_BF16X2, OUT_F32 = 0, 1, 2


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    lib = ctypes.CDLL(LIB_PATH)
    vp, i = ctypes.c_void_p, ctypes.c_int
    lib.laya_b200_gemm.restype = i
    lib.laya_b200_gemm.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, i, i, i, i, vp, vp, vp, i, i, vp, i]
    return lib


def P(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def gemm(L, A, W, out, M, N, K, planes=1, epi=EPI_STORE, out_mode=OUT_F32, act=0, bn=256, resid=None,
         bias=None, cos=None, sin=None, pos=None, rope_cols=0, geglu_I=0):
    torch.cuda.synchronize()
    rc = L.laya_b200_gemm(P(A), P(W), P(out), P(resid), P(bias), M, N, K, planes, epi, out_mode, act, bn,
                          P(cos), P(sin), P(pos), rope_cols, geglu_I, None, 1)
    assert rc == 0, "laya_b200_gemm returned %d" % rc


def rel(a, b):
    return float((a.double() - b.double()).abs().max() / b.double().abs().max().clamp_min(1e-30))


def split(x):
    hi = x.to(torch.bfloat16)
    lo = (x - hi.float()).to(torch.bfloat16)
    return torch.stack([hi, lo]).contiguous()


@pytest.mark.parametrize("bn", [128, 256, 512])
@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (127, 512, 1024), (300, 1024, 72), (1024, 3072, 1024),
                                   (520, 1024, 2624), (4096, 768, 1152), (600, 1152, 1024), (2000, 640, 320)])
def test_store_f32(L, bn, M, N, K):
    """N = 1152 and 640 end in a half-filled 256-column tile."""
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.02 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    out = torch.full((M, N), float("nan"), device="cuda")
    gemm(L, A, W, out, M, N, K, bn=bn)
    ref = A.double() @ W.double().T
    assert rel(out, ref) < 1e-4


@pytest.mark.parametrize("bn", [128, 256, 512])
@pytest.mark.parametrize("M,N,K", [(200, 1024, 1024), (512, 3072, 1024), (333, 1024, 4096)])
def test_split_bf16_parity(L, bn, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(11 + M)
    A32 = torch.randn(M, K, device="cuda", generator=g)
    W32 = 0.02 * torch.randn(N, K, device="cuda", generator=g)
    out = torch.empty((M, N), device="cuda")
    gemm(L, split(A32), split(W32), out, M, N, K, planes=2, bn=bn)
    ref = A32.double() @ W32.double().T
    err = rel(out, ref)
    assert err < 5e-5, err
    # the same data through one bf16 product is two orders of magnitude worse
    out1 = torch.empty((M, N), device="cuda")
    gemm(L, A32.bfloat16().contiguous(), W32.bfloat16().contiguous(), out1, M, N, K, planes=1, bn=bn)
    assert rel(out1, ref) > 20 * err


@pytest.mark.parametrize("act", [0, 1, 2])
def test_bias_act_bf16(L, act):
    M, N, K = 700, 4096, 1024
    g = torch.Generator(device="cuda").manual_seed(act)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.05 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    b = 0.1 * torch.randn(N, device="cuda", generator=g)
    out = torch.empty((M, N), device="cuda", dtype=torch.bfloat16)
    gemm(L, A, W, out, M, N, K, out_mode=OUT_BF16, act=act, bias=b)
    ref = A.double() @ W.double().T + b.double()
    ref = [ref, torch.relu(ref), torch.nn.functional.gelu(ref)][act]
    assert rel(out.float(), ref) < 1e-2


def test_bf16x2_planes(L):
    M, N, K = 400, 1024, 1024
    g = torch.Generator(device="cuda").manual_seed(5)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.02 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    out = torch.empty((2, M, N), device="cuda", dtype=torch.bfloat16)
    gemm(L, A, W, out, M, N, K, out_mode=OUT_BF16X2)
    ref = A.double() @ W.double().T
    assert rel(out[0].float() + out[1].float(), ref) < 1e-4


@pytest.mark.parametrize("bn", [128, 256, 512])
def test_residual(L, bn):
    M, N, K = 777, 1024, 2624
    g = torch.Generator(device="cuda").manual_seed(9)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.02 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    b = torch.randn(N, device="cuda", generator=g)
    x0 = 10 * torch.randn(M, N, device="cuda", generator=g)
    x = x0.clone()
    gemm(L, A, W, None, M, N, K, epi=EPI_RESID, resid=x, bias=b, bn=bn)
    ref = x0.double() + A.double() @ W.double().T + b.double()
    assert rel(x, ref) < 1e-6 * 100


def rope_tables(max_pos, theta):
    inv = 1.0 / (theta ** (torch.arange(0, 64, 2, dtype=torch.float32) / 64))
    f = torch.arange(max_pos, dtype=torch.float32)[:, None] * inv[None, :]
    return torch.cos(f).cuda().contiguous(), torch.sin(f).cuda().contiguous()


@pytest.mark.parametrize("bn", [128, 256, 512])
def test_rope(L, bn):
    D, M, K = 256, 300, 256
    N = 3 * D
    g = torch.Generator(device="cuda").manual_seed(3)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.05 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    pos = torch.randint(0, 512, (M,), device="cuda", generator=g, dtype=torch.int32)
    cos, sin = rope_tables(512, 10000.0)
    out = torch.empty((M, N), device="cuda")
    gemm(L, A, W, out, M, N, K, epi=EPI_ROPE, cos=cos, sin=sin, pos=pos, rope_cols=2 * D, bn=bn)
    y = (A.double() @ W.double().T)
    c = cos[pos.long()].double().repeat(1, 2)
    s = sin[pos.long()].double().repeat(1, 2)
    ref = y.clone()
    for part in range(2):
        for h in range(D // 64):
            sl = slice(part * D + h * 64, part * D + h * 64 + 64)
            x = y[:, sl]
            rot = torch.cat([-x[:, 32:], x[:, :32]], dim=1)
            ref[:, sl] = x * c + rot * s
    assert rel(out, ref) < 1e-4


def interleave_geglu(W, I, group=64):
    """[2I, K] (input rows then gate rows) -> groups of 64 input rows followed by their gate rows."""
    parts = []
    for j in range(0, I, group):
        g = min(group, I - j)
        parts.append(W[j:j + g])
        parts.append(W[I + j:I + j + g])
    return torch.cat(parts).contiguous()


@pytest.mark.parametrize("I,bn", [(2624, 256), (1152, 256), (2624, 128), (192, 256), (2624, 512), (192, 512)])
def test_geglu(L, I, bn):
    M, K = 513, 1024
    g = torch.Generator(device="cuda").manual_seed(I)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.03 * torch.randn(2 * I, K, device="cuda", generator=g)).bfloat16()
    out = torch.empty((M, I), device="cuda")
    gemm(L, A, interleave_geglu(W, I), out, M, 2 * I, K, epi=EPI_GEGLU, geglu_I=I, bn=bn)
    y = A.double() @ W.double().T
    ref = torch.nn.functional.gelu(y[:, :I]) * y[:, I:]
    assert rel(out, ref) < 1e-4


def test_geglu_gelu_error_bound(L):
    """The epilogue's GELU (Abramowitz & Stegun 7.1.26 form of erfc, one reciprocal and one 2^x)
    against the exact-erf GELU in fp64, isolated: A row m is s_m e_0 (s_m a power of two) and the
    interleaved weight rows put x_n in column 0 of input row n and 1 in column 0 of its gate row, so
    the accumulator holds y = s_m x_n and the gate s_m exactly; out / s_m = gelu(y) as computed by the
    kernel, for |y| up to 12 on a dense bf16 grid. Bound: 1e-6 absolute plus 2^-22 relative (fp32
    rounding of y * Phi(y) near |y| = 12 alone is up to 4.8e-7)."""
    I, K = 2624, 64
    xs = torch.linspace(-1.5, 1.5, I, device="cuda").bfloat16()
    scales = [2.0 ** e for e in range(-4, 4)]
    M = len(scales)
    A = torch.zeros(M, K, device="cuda")
    for m, sc in enumerate(scales):
        A[m, 0] = sc
    A = A.bfloat16()
    W = torch.zeros(2 * I, K, device="cuda")
    W[:I, 0] = xs.float()
    W[I:, 0] = 1.0
    W = W.bfloat16()
    out = torch.empty((M, I), device="cuda")
    gemm(L, A, interleave_geglu(W, I), out, M, 2 * I, K, epi=EPI_GEGLU, geglu_I=I, bn=256)
    sc = torch.tensor(scales, device="cuda", dtype=torch.float64)[:, None]
    y = sc * xs.double()[None, :]
    ref = 0.5 * y * (1.0 + torch.erf(y / math.sqrt(2.0)))
    err = (out.double() / sc - ref).abs()
    assert float((err - (1e-6 + 2.0 ** -22 * ref.abs())).max()) <= 0.0, float(err.max())


# ---------------------------------------------------------------- split-K (small M)
@pytest.fixture(scope="module")
def LS(L):
    vp, i = ctypes.c_void_p, ctypes.c_int
    L.laya_b200_gemm_splitk.restype = i
    L.laya_b200_gemm_splitk.argtypes = [vp, vp, vp, vp, vp, i, i, i, i, i, i, i, i, vp, vp, vp, i, i, i, vp, i]
    return L


def gemm_split(L, splits, A, W, out, M, N, K, planes=1, epi=EPI_STORE, out_mode=OUT_F32, act=0, bn=128, resid=None,
               bias=None, cos=None, sin=None, pos=None, rope_cols=0, geglu_I=0):
    torch.cuda.synchronize()
    rc = L.laya_b200_gemm_splitk(P(A), P(W), P(out), P(resid), P(bias), M, N, K, planes, epi, out_mode, act, bn,
                                 P(cos), P(sin), P(pos), rope_cols, geglu_I, splits, None, 1)
    assert rc == 0, "laya_b200_gemm_splitk returned %d" % rc


@pytest.mark.parametrize("splits", [2, 3, 4, 8])
@pytest.mark.parametrize("bn", [128, 256])
def test_splitk_store_and_resid(LS, splits, bn):
    M, N, K = 300, 1024, 2624
    g = torch.Generator(device="cuda").manual_seed(splits)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    W = (0.02 * torch.randn(N, K, device="cuda", generator=g)).bfloat16()
    b = torch.randn(N, device="cuda", generator=g)
    ref = A.double() @ W.double().T
    out = torch.full((M, N), float("nan"), device="cuda")
    gemm_split(LS, splits, A, W, out, M, N, K, bn=bn)
    assert rel(out, ref) < 1e-4
    out2 = torch.full((M, N), float("nan"), device="cuda")
    gemm_split(LS, splits, A, W, out2, M, N, K, bn=bn)
    assert torch.equal(out, out2)  # slice sums in fixed order: bitwise repeatable
    x0 = torch.randn(M, N, device="cuda", generator=g)
    x = x0.clone()
    gemm_split(LS, splits, A, W, None, M, N, K, epi=EPI_RESID, resid=x, bias=b, bn=bn)
    assert rel(x, x0.double() + ref + b.double()) < 1e-5


@pytest.mark.parametrize("splits", [2, 4])
def test_splitk_epilogues(LS, splits):
    M, K, I = 513, 1024, 1152
    g = torch.Generator(device="cuda").manual_seed(40 + splits)
    A = torch.randn(M, K, device="cuda", generator=g).bfloat16()
    # GeGLU
    W = (0.03 * torch.randn(2 * I, K, device="cuda", generator=g)).bfloat16()
    out = torch.empty((M, I), device="cuda")
    gemm_split(LS, splits, A, interleave_geglu(W, I), out, M, 2 * I, K, epi=EPI_GEGLU, geglu_I=I)
    y = A.double() @ W.double().T
    assert rel(out, torch.nn.functional.gelu(y[:, :I]) * y[:, I:]) < 1e-4
    # RoPE
    D = 256
    Wq = (0.05 * torch.randn(3 * D, K, device="cuda", generator=g)).bfloat16()
    pos = torch.randint(0, 512, (M,), device="cuda", generator=g, dtype=torch.int32)
    cos, sin = rope_tables(512, 160000.0)
    outq = torch.empty((M, 3 * D), device="cuda")
    gemm_split(LS, splits, A, Wq, outq, M, 3 * D, K, epi=EPI_ROPE, cos=cos, sin=sin, pos=pos, rope_cols=2 * D)
    outq1 = torch.empty((M, 3 * D), device="cuda")
    gemm(LS, A, Wq, outq1, M, 3 * D, K, epi=EPI_ROPE, cos=cos, sin=sin, pos=pos, rope_cols=2 * D, bn=128)
    assert rel(outq, outq1) < 1e-5
    # bias + GELU to bf16 hi/lo planes, fp32-parity operands
    A32 = torch.randn(M, K, device="cuda", generator=g)
    W32 = 0.02 * torch.randn(1024, K, device="cuda", generator=g)
    bb = 0.1 * torch.randn(1024, device="cuda", generator=g)
    o2 = torch.empty((2, M, 1024), device="cuda", dtype=torch.bfloat16)
    gemm_split(LS, splits, split(A32), split(W32), o2, M, 1024, K, planes=2, out_mode=OUT_BF16X2, act=2, bias=bb)
    refg = torch.nn.functional.gelu(A32.double() @ W32.double().T + bb.double())
    assert rel(o2[0].float() + o2[1].float(), refg) < 1e-4
