"""Debug bounds mode, host side (no GPU): the packing checker that the engine runs on every pass's
metadata block before uploading it in debug bounds mode, exercised through the host-only entry
laya_pack_check on random batches (valid blocks pass) and on blocks with one map broken on purpose in
host memory (each is caught by the check that guards that map); the debug-bounds build exports the
same ABI and says so."""
import ctypes
import os
import re

import numpy as np
import pytest

from layamd_b200 import build as lb
from layamd_b200 import load_lib
from layamd_b200.synthetic import synth, workloads

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
IP = ctypes.POINTER(ctypes.c_int)

# map broken by `corrupt` -> number of the check that must reject it (engine.cpp check_pass_meta)
BROKEN = {1: 2, 2: 3, 3: 4, 4: 6, 5: 7, 6: 8, 7: 11, 8: 13}


def pack_check(L, arch, qs, pass_tokens, max_seqs=4096, corrupt=0):
    lens, ids, nmark, markers, qtypes = workloads.flatten(qs)
    p = lambda a: (a if a.size else np.zeros(1, np.int32)).ctypes.data_as(IP)  # noqa: E731
    return L.laya_pack_check(arch.max_len, arch.vocab, arch.pad_id, pass_tokens, max_seqs, len(qs), p(lens), p(ids),
                             p(nmark), p(markers), p(qtypes), corrupt)


@pytest.mark.parametrize("seed", range(6))
def test_random_batches_pass_the_packing_check(seed):
    L = load_lib()
    rng = np.random.default_rng(seed)
    a = synth.ARCHS["tiny"] if seed % 2 else synth.ARCHS["large"]
    qs = workloads.mixed(a, int(rng.integers(1, 80)), seed=100 + seed, kmax=int(rng.integers(1, 40)))
    for pass_tokens in (a.max_len, 4 * a.max_len, 65536):
        n = pack_check(L, a, qs, pass_tokens, max_seqs=int(rng.integers(1, 50)))
        assert n >= 1, n


def test_benchmark_batches_pass_the_packing_check():
    L = load_lib()
    for name, qs in (("large", workloads.c2(synth.ARCHS["large"])), ("large", workloads.seq512(synth.ARCHS["large"])),
                     ("large1024", workloads.c4(synth.ARCHS["large1024"])), ("base", workloads.c3(synth.ARCHS["base"]))):
        assert pack_check(L, synth.ARCHS[name], qs, 131072) == 1


@pytest.mark.parametrize("which,check", sorted(BROKEN.items()))
def test_each_broken_map_is_caught(which, check):
    L = load_lib()
    a = synth.ARCHS["tiny"]
    qs = workloads.mixed(a, 9, seed=7, kmax=5)
    assert pack_check(L, a, qs, 4096) >= 1
    assert pack_check(L, a, qs, 4096, corrupt=which) == -100 - check


def test_invalid_batches_are_refused_before_packing():
    L = load_lib()
    a = synth.ARCHS["tiny"]
    q = workloads.mixed(a, 2, seed=3, kmax=3)
    assert pack_check(L, a, [dict(q[0], ids=[a.vocab] + q[0]["ids"][1:])], 4096) == -1  # id past the vocabulary
    assert pack_check(L, a, [dict(q[0], qtype=3)], 4096) == -1
    assert pack_check(L, a, [dict(q[0], markers=[len(q[0]["ids"])])], 4096) == -1


def test_debug_bounds_build_exports_the_same_abi():
    if not os.path.exists(lb.LIB_DBG):
        pytest.skip("debug bounds build absent (python -m layamd_b200.build --debug-bounds)")
    src = re.sub(r"/\*.*?\*/", "", open(os.path.join(ROOT, "include", "laya_api.h")).read(), flags=re.S)
    names = sorted(set(re.findall(r"\b(laya_\w+)\s*\(", src)))
    dbg = ctypes.CDLL(lb.LIB_DBG)
    assert not [n for n in names if not hasattr(dbg, n)]
    assert dbg.laya_debug_bounds_build() == 1
    assert load_lib().laya_debug_bounds_build() == 0
