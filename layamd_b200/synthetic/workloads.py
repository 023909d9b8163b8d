"""Seeded synthetic inputs of the benchmark configurations, for the tests and the benchmarks (token
ids and option markers only; nothing here computes the model).

Every question is a dict {ids, markers, qtype} in the reference ABI's terms
(src/laya_api.h:6-9): token ids of one sequence, option-marker positions within it, question type
(0 choice, 1 score, 2 noul/yes-no, ref/rl_common.py:17). Each sequence starts with CLS, ends with
SEP and carries the mask token at its markers, like ref/rl_common.py:47-77 lays them out.
"""
import math
import random

import numpy as np


def _question(rng, L, k, qtype, arch, id_lo=5, id_hi=None):
    id_hi = id_hi or arch.vocab
    ids = rng.integers(id_lo, id_hi, size=L).astype(np.int64)
    hi = max(1, min(L - 1, 1 + 4 * k))
    pool = np.arange(1, hi + 1) if L > 1 else np.array([0])
    k = min(k, len(pool))
    markers = np.sort(rng.choice(pool, size=k, replace=False)) if L > 1 else np.zeros(1, np.int64)
    ids[0] = arch.cls_id
    if L > 1:
        ids[L - 1] = arch.sep_id
    ids[markers] = arch.mask_id
    return {"ids": ids.tolist(), "markers": markers.tolist(), "qtype": int(qtype)}


def c1(arch, L=512, seed=0):
    """Batch 1, one 3-option choice question, markers at 16/24/32."""
    rng = np.random.default_rng(seed)
    ids = rng.integers(5, arch.vocab, size=L).astype(np.int64)
    ids[0], ids[L - 1] = arch.cls_id, arch.sep_id
    markers = [16, 24, 32]
    ids[markers] = arch.mask_id
    return [{"ids": ids.tolist(), "markers": markers, "qtype": 0}]


def c2(arch, states=64, seed=1):
    """64 states with L ~ U[32,512]; per state a choice (k ~ U{2..5}), a 3-level score and a yes/no."""
    r = random.Random(seed)
    lens = [r.randint(32, 512) for _ in range(states)]
    rng = np.random.default_rng(seed)
    qs = []
    for L in lens:
        qs.append(_question(rng, L, int(rng.integers(2, 6)), 0, arch))
        qs.append(_question(rng, L, 3, 1, arch))
        qs.append(_question(rng, L, 2, 2, arch))
    return qs


def seq512(arch, B=128, L=512, seed=5):
    """Fixed length: B choice questions of exactly L tokens with 3 options each (the metric's seq512)."""
    rng = np.random.default_rng(seed)
    return [_question(rng, L, 3, 0, arch) for _ in range(B)]


def c3(arch, B=128, seed=3):
    """mmBERT-base shapes: L ~ U[64,1024], ids over the whole vocabulary, one 3-option choice each."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(64, 1025, size=B)
    return [_question(rng, int(L), 3, 0, arch, id_lo=0) for L in lens]


def c4(arch, B=256, seed=4):
    """L log-uniform in [128,1024]; question types cycle choice/score/noul; 2-6 options (noul: 2)."""
    rng = np.random.default_rng(seed)
    lens = np.rint(np.exp(rng.uniform(math.log(128), math.log(1024), size=B))).astype(int)
    qs = []
    for b, L in enumerate(lens):
        qt = b % 3
        k = 2 if qt == 2 else int(rng.integers(2, 7))
        qs.append(_question(rng, int(L), k, qt, arch))
    return qs


def mixed(arch, B, seed, max_len=None, kmax=6):
    """Random lengths in [1, max_len] and 1..kmax options: edge-case coverage for parity tests."""
    rng = np.random.default_rng(seed)
    max_len = max_len or arch.max_len
    qs = []
    for b in range(B):
        L = int(rng.integers(1, max_len + 1))
        k = int(rng.integers(1, kmax + 1))
        qs.append(_question(rng, L, k, int(rng.integers(0, 3)), arch))
    return qs


def n_tokens(qs):
    return sum(len(q["ids"]) for q in qs)


def flatten(qs):
    """ABI arrays (lens, ids, nmark, markers, qtypes) as int32 numpy arrays."""
    lens = np.array([len(q["ids"]) for q in qs], np.int32)
    ids = np.array([t for q in qs for t in q["ids"]], np.int32)
    nmark = np.array([len(q["markers"]) for q in qs], np.int32)
    markers = np.array([m for q in qs for m in q["markers"]], np.int32)
    qtypes = np.array([q["qtype"] for q in qs], np.int32)
    return lens, ids, nmark, markers, qtypes
