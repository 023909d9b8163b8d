"""Host-side checks that need no GPU: the library loads and exports every symbol include/laya_api.h
declares, the load-error path, and the pass packer against a restatement of the reference's packing
rule (src/engine.hip:489-505) including the -1 validation contract, and the GEMM planner's choices at
the measured shapes."""
import ctypes
import os
import re

import numpy as np
import pytest

from layamd_b200 import LIB_PATH, load_lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
IP = ctypes.POINTER(ctypes.c_int)


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "laya_api.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(laya_\w+)\s*\(", src)))


def test_header_has_reference_abi():
    names = declared_symbols()
    for n in ["laya_create", "laya_forward_batch", "laya_forward", "laya_n_act", "laya_max_len", "laya_max_markers",
              "laya_temperature", "laya_prof_report", "laya_prof_reset", "laya_tune_all"]:
        assert n in names


def test_library_exports_every_declared_symbol():
    assert os.path.exists(LIB_PATH), "build the library first (python -m layamd_b200.build)"
    lib = ctypes.CDLL(LIB_PATH)
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing
    load_lib()  # every signature binds


def test_create_missing_dir_returns_null():
    L = load_lib()
    assert not L.laya_create(b"/nonexistent/laya_model_dir")
    assert L.laya_n_act(None) == 0 and L.laya_forward_batch(None, 0, None, None, None, None, None, None, None) == -1


def plan_reference(lens, nmark, pass_tokens, max_seqs, max_gathered):
    """Greedy in-order packing: a pass takes questions while rows <= pass_tokens, questions <= max_seqs
    and gathered rows (markers + one CLS row each) <= max_gathered."""
    passes, b0, B = [], 0, len(lens)
    while b0 < B:
        n = T = KT = 0
        while b0 + n < B and n < max_seqs:
            b = b0 + n
            if n > 0 and (T + lens[b] > pass_tokens or KT + nmark[b] + n + 1 > max_gathered):
                break
            T += lens[b]
            KT += nmark[b]
            n += 1
        passes.append((b0, n, T))
        b0 += n
    return passes


def run_plan(max_len, pass_tokens, max_seqs, lens, nmark, markers):
    L = load_lib()
    lens = np.asarray(lens, np.int32)
    nmark = np.asarray(nmark, np.int32)
    markers = np.asarray(markers, np.int32)
    cap = len(lens) + 1
    f, c, r = (np.zeros(cap, np.int32) for _ in range(3))
    p = lambda a: a.ctypes.data_as(IP)  # noqa: E731
    n = L.laya_plan_passes_cfg(max_len, pass_tokens, max_seqs, len(lens), p(lens), p(nmark), p(markers if markers.size
                               else np.zeros(1, np.int32)), cap, p(f), p(c), p(r))
    return n, list(zip(f[:max(n, 0)].tolist(), c[:max(n, 0)].tolist(), r[:max(n, 0)].tolist()))


@pytest.mark.parametrize("seed", range(6))
def test_packer_matches_reference_rule(seed):
    rng = np.random.default_rng(seed)
    B = int(rng.integers(1, 200))
    max_len = 512
    lens = rng.integers(1, max_len + 1, B)
    nmark = rng.integers(1, 9, B)
    nmark = np.minimum(nmark, lens)
    markers = np.concatenate([rng.choice(l, k, replace=False) for l, k in zip(lens, nmark)])
    pass_tokens = int(rng.choice([512, 1024, 4096, 131072]))
    max_seqs = int(rng.choice([1, 3, 128, 4096]))
    n, got = run_plan(max_len, pass_tokens, max_seqs, lens, nmark, markers)
    want = plan_reference(lens.tolist(), nmark.tolist(), pass_tokens, max_seqs, max(pass_tokens // 4, 512))
    assert n == len(want) and got == want
    assert sum(c for _, c, _ in got) == B


def test_packer_rejects_invalid_batches():
    ok = dict(lens=[10, 20], nmark=[2, 3], markers=[1, 2, 0, 5, 19])
    assert run_plan(512, 1024, 128, **ok)[0] == 1
    for bad in [dict(ok, lens=[0, 20]), dict(ok, lens=[10, 513]), dict(ok, nmark=[0, 5], markers=[0, 1, 2, 5, 19]),
                dict(ok, markers=[1, 10, 0, 5, 19]), dict(ok, markers=[1, 2, 0, 5, -1]),
                dict(lens=[300], nmark=[256], markers=[1] * 256)]:
        assert run_plan(512, 1024, 128, **bad)[0] == -1


def plan(L, M, N, K, parity=0, ln=0, sms=148, pairs=74):
    bn, splits = ctypes.c_int(0), ctypes.c_int(0)
    assert L.laya_plan_gemm(M, N, K, parity, sms, pairs, ln, ctypes.byref(bn), ctypes.byref(splits)) == 0
    return bn.value, splits.value


def test_gemm_planner_at_the_measured_shapes():
    """The engine's per-launch GEMM plan (tile, K slices) on a 148-SM B200 with 74 co-resident CTA
    pairs, at the ModernBERT-large shapes whose choices were measured: 512 rows (batch 1) and the
    52,287-row C2 pass."""
    L = load_lib()
    # batch 1, 512 rows: QKV and K = 1024 stores stay whole on 128 x 128 tiles; GeGLU takes one wave
    # of 128 x 256 tiles; the residual GEMMs followed by a bias-free LayerNorm split 4 ways (their
    # reduce kernel takes the LayerNorm over), as does the head's K = 4096 FFN-2 (bias LayerNorm: no
    # credit, still worth 4 slices)
    assert plan(L, 512, 3072, 1024) == (128, 1)
    assert plan(L, 512, 5248, 1024) == (256, 1)
    assert plan(L, 512, 1024, 1024, ln=1) == (128, 4)
    assert plan(L, 512, 1024, 2624, ln=1) == (128, 4)
    assert plan(L, 512, 1024, 4096) == (128, 4)
    # without the LayerNorm credit the K = 1024 residual GEMM stays whole
    assert plan(L, 512, 1024, 1024) == (128, 1)
    # fp32-parity mode: three products per K block make the K loops long enough to split without it
    assert plan(L, 512, 1024, 1024, parity=1) == (128, 4)
    # C2 pass: every encoder GEMM on CTA-pair 256 x 256 tiles, whole K
    for N, K in ((3072, 1024), (1024, 1024), (5248, 1024), (1024, 2624)):
        assert plan(L, 52287, N, K, ln=1) == (512, 1)
    # 4096 rows: too few 256 x 256 tiles to fill the pairs twice, so one-CTA tiles by whole waves
    assert plan(L, 4096, 1024, 1024) == (256, 1)
    assert plan(L, 52287, 1024, 1024, pairs=0) == (256, 1)  # no pair kernel on the device
    # bad arguments
    bn, splits = ctypes.c_int(0), ctypes.c_int(0)
    assert L.laya_plan_gemm(0, 1024, 1024, 0, 148, 74, 0, ctypes.byref(bn), ctypes.byref(splits)) == -1
