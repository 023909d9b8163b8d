"""Encoder attention kernels through the C ABI (laya_b200_attention) against an fp32 PyTorch reference.

The tcgen05 kernel (impl 0: 128-query tiles, S and O in tensor memory) and the mma.sync kernel
(impl 1) must both match softmax(q k^T / 8) v per head within each packed sequence, with the
bidirectional band |q - k| <= window on sliding layers (transformers' sliding-window overlay, as the
reference's k_flash_wmma applies it, src/kernels.hip:154-242). bf16 inputs and outputs, fp32 softmax:
tolerance max|a - b| / max|b| < 1e-2 per case.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def L():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from layamd_b200 import load_lib
    return load_lib()


def reference(qkv, lens, H, window):
    D = 64 * H
    out = torch.zeros(qkv.shape[0], D, dtype=torch.float32, device=qkv.device)
    off = 0
    for n in lens:
        x = qkv[off:off + n].float()
        q = x[:, :D].view(n, H, 64).transpose(0, 1)
        k = x[:, D:2 * D].view(n, H, 64).transpose(0, 1)
        v = x[:, 2 * D:].view(n, H, 64).transpose(0, 1)
        s = q @ k.transpose(1, 2) * 0.125
        if window:
            i = torch.arange(n, device=qkv.device)
            s = s.masked_fill((i[:, None] - i[None, :]).abs() > window, float("-inf"))
        out[off:off + n] = (torch.softmax(s, -1) @ v).transpose(0, 1).reshape(n, D)
        off += n
    return out


def run(L, qkv, lens, H, window, impl):
    rows = qkv.shape[0]
    out = torch.zeros(rows, 64 * H, dtype=torch.bfloat16, device=qkv.device)
    la = np.asarray(lens, dtype=np.int32)
    rc = L.laya_b200_attention(ctypes.c_void_p(qkv.data_ptr()), ctypes.c_void_p(out.data_ptr()), rows, len(lens),
                               la.ctypes.data_as(ctypes.POINTER(ctypes.c_int)), H, window, impl, None, 1)
    assert rc == 0, "laya_b200_attention returned %d" % rc
    return out


def rel(a, b):
    return ((a.float() - b.float()).abs().max() / b.float().abs().max()).item()


def make_qkv(lens, H, seed, extra_rows=200, scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rows = sum(lens) + extra_rows  # finite filler rows after the last sequence
    return (scale * torch.randn(rows, 3 * 64 * H, device="cuda", generator=g)).bfloat16()


LENS = [1, 17, 64, 127, 128, 129, 255, 300, 512, 513, 1024]


@pytest.mark.parametrize("window", [0, 64])
@pytest.mark.parametrize("impl", [0, 1])
def test_ragged_sequences(L, window, impl):
    H = 4
    qkv = make_qkv(LENS, H, seed=1 + window)
    ref = reference(qkv, LENS, H, window)
    out = run(L, qkv, LENS, H, window, impl)
    T = sum(LENS)
    assert rel(out[:T], ref[:T]) < 1e-2
    assert out[T:].abs().max().item() == 0.0  # rows past the sequences are never written


@pytest.mark.parametrize("window", [0, 64])
def test_tc_matches_mma_sync_full_width(L, window):
    """16 heads (ModernBERT-large width), the C2 length range."""
    rng = np.random.default_rng(5)
    lens = [int(x) for x in rng.integers(32, 513, size=24)]
    H = 16
    qkv = make_qkv(lens, H, seed=7)
    a = run(L, qkv, lens, H, window, 0)
    b = run(L, qkv, lens, H, window, 1)
    ref = reference(qkv, lens, H, window)
    T = sum(lens)
    assert rel(a[:T], ref[:T]) < 1e-2
    assert rel(a[:T], b[:T]) < 1e-2


@pytest.mark.parametrize("window", [0, 64])
def test_growing_scores_exercise_the_running_max(L, window):
    """Keys grow along the sequence so each 128-key chunk raises the row max by far more than 2^8:
    the tensor-memory O accumulator must be rescaled chunk after chunk (inside the +-64 band too)."""
    lens = [1000, 700]
    H = 2
    qkv = make_qkv(lens, H, seed=11, scale=0.5).float()
    D = 64 * H
    off = 0
    for n in lens:
        ramp = torch.linspace(0.2, 20.0, n, device="cuda")[:, None]
        qkv[off:off + n, D:2 * D] *= ramp
        qkv[off:off + n, :D] = qkv[off:off + n, :D].abs() + 1.0
        qkv[off:off + n, D:2 * D] = qkv[off:off + n, D:2 * D].abs()
        off += n
    qkv = qkv.bfloat16()
    ref = reference(qkv, lens, H, window)
    T = sum(lens)
    for impl in (0, 1):
        out = run(L, qkv, lens, H, window, impl)
        assert rel(out[:T], ref[:T]) < 1e-2, impl


def test_repeated_calls_are_bitwise_stable(L):
    lens = [300, 77, 512]
    H = 16
    qkv = make_qkv(lens, H, seed=3)
    a = run(L, qkv, lens, H, 64, 0)
    b = run(L, qkv, lens, H, 64, 0)
    assert torch.equal(a, b)
