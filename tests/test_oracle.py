"""Pins the numpy oracle (oracle/model.py) to the reference's own PyTorch path through the golden
fixtures in tests/golden/ (made by tests/golden/make_golden.py from ref/rl_common.py + transformers).

Tolerances: both sides compute in fp32 on the CPU and differ only in reduction order, so hidden
states agree to max|a-b|/max|b| < 2e-5 per layer and logits / act logits to 1e-5 absolute (relative
for the act head, whose logits are larger).
"""
import os

import numpy as np
import pytest

from oracle import model as om
from layamd_b200.synthetic import synth

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


def questions_of(g):
    qs, io, mo = [], 0, 0
    for L, k, qt in zip(g["lens"], g["nmark"], g["qtypes"]):
        qs.append({"ids": g["ids"][io:io + L].tolist(), "markers": g["markers"][mo:mo + k].tolist(), "qtype": int(qt)})
        io += L
        mo += k
    return qs


def check_fingerprint(weights, name):
    fp = np.load(os.path.join(GOLD, name))
    for k in fp.files:
        v = np.asarray(weights[k], np.float64).ravel()
        got = np.array([v.sum(), (v * v).sum(), v[0]])
        assert np.allclose(got, fp[k], rtol=1e-9, atol=1e-9), k


@pytest.fixture(scope="module")
def tiny():
    ck = synth.checkpoint("tiny", 0)
    w = synth.load_weights(ck)
    check_fingerprint(w, "tiny_weights_fp.npz")
    return om.Oracle(w, synth.load_arch(ck))


@pytest.mark.parametrize("case", ["tiny_mixed", "tiny_k1", "tiny_full"])
def test_tiny_layers(tiny, case):
    g = np.load(os.path.join(GOLD, case + ".npz"))
    qs = questions_of(g)
    lo, ac, caps = tiny.forward_batch(qs, capture=True)
    assert np.abs(lo - g["logits"]).max() < 1e-5
    assert np.abs(ac - g["act"]).max() < 1e-5 * max(1.0, np.abs(g["act"]).max())
    for key in ["emb", "final_norm"] + ["enc%d" % i for i in range(4)] + ["head0", "head1"]:
        mine = np.concatenate([c[key] for c in caps])
        assert rel(mine, g["t_" + key]) < 2e-5, key


@pytest.mark.slow
@pytest.mark.parametrize("case", ["large_c1", "large_multi"])
def test_large(case):
    ck = synth.checkpoint("large", 0)
    w = synth.load_weights(ck)
    check_fingerprint(w, "large_weights_fp.npz")
    o = om.Oracle(w, synth.load_arch(ck))
    g = np.load(os.path.join(GOLD, case + ".npz"))
    qs = questions_of(g)
    lo, ac, caps = o.forward_batch(qs, capture=True)
    assert np.abs(lo - g["logits"]).max() < 2e-5
    assert np.abs(ac - g["act"]).max() < 2e-5 * max(1.0, np.abs(g["act"]).max())
    rows = g["sample_rows"]
    for key in ["emb", "final_norm", "head0", "head1"] + ["enc%d" % i for i in range(28)]:
        norms = np.concatenate([np.linalg.norm(c[key], axis=-1) for c in caps])
        assert rel(norms, g["n_" + key]) < 2e-5, key
        assert rel(caps[0][key][rows], g["s_" + key]) < 5e-5, key


@pytest.mark.slow
@pytest.mark.parametrize("arch,case,layers", [("base", "base_c3", 22), ("large1024", "large1024_c4", 28)])
def test_other_configurations(arch, case, layers):
    """C3 (mmBERT-base: vocabulary 256,000, pad id 0, 22 layers, d 768; a 987-token question) and C4
    (ModernBERT-large at context 1024: RoPE positions up to 1020, global attention over 1021 keys),
    each in a padded batch with shorter questions, against the reference's own path."""
    ck = synth.checkpoint(arch, 0)
    w = synth.load_weights(ck)
    check_fingerprint(w, arch + "_weights_fp.npz")
    o = om.Oracle(w, synth.load_arch(ck))
    g = np.load(os.path.join(GOLD, case + ".npz"))
    qs = questions_of(g)
    assert max(len(q["ids"]) for q in qs) > 900
    lo, ac, caps = o.forward_batch(qs, capture=True)
    assert np.abs(lo - g["logits"]).max() < 2e-5
    assert np.abs(ac - g["act"]).max() < 2e-5 * max(1.0, np.abs(g["act"]).max())
    rows = g["sample_rows"]
    for key in ["emb", "final_norm", "head0", "head1"] + ["enc%d" % i for i in range(layers)]:
        norms = np.concatenate([np.linalg.norm(c[key], axis=-1) for c in caps])
        assert rel(norms, g["n_" + key]) < 2e-5, key
        assert rel(caps[0][key][rows], g["s_" + key]) < 5e-5, key


def test_rope_tables_match_transformers_formula():
    cos, sin = om.rope_tables(8, 10000.0)
    inv = 1.0 / (10000.0 ** (np.arange(0, 64, 2) / 64))
    f = np.arange(8)[:, None] * inv[None, :]
    assert np.abs(cos[:, :32] - np.cos(f)).max() < 1e-6
    assert np.abs(sin[:, 32:] - np.sin(f)).max() < 1e-6


def test_c2_golden_inputs_are_the_benchmark_batch():
    """The reference logits of the whole C2 batch were made on exactly the inputs the benchmark and
    the GPU test generate (lengths, option counts, marker positions, token-id checksum)."""
    from layamd_b200.synthetic import workloads
    g = np.load(os.path.join(GOLD, "large_c2_logits.npz"))
    lens, ids, nmark, markers, qtypes = workloads.flatten(workloads.c2(synth.ARCHS["large"], seed=1))
    assert (lens == g["lens"]).all() and (nmark == g["nmark"]).all() and (qtypes == g["qtypes"]).all()
    assert (markers == g["markers"]).all() and int(ids.astype(np.int64).sum()) == int(g["ids_sum"])
    assert g["logits"].shape == (int(nmark.sum()),) and g["act"].shape == (192, 2)
    assert np.isfinite(g["logits"]).all()


@pytest.mark.parametrize("arch,workload,case,B", [("base", "c3", "base_c3_logits", 128),
                                                  ("large1024", "c4", "large1024_c4_logits", 256),
                                                  ("large", "seq512", "large_seq512_logits", 128)])
def test_whole_batch_golden_inputs_are_the_benchmark_batches(arch, workload, case, B):
    """The same for the reference logits of the whole C3, C4 and fixed-length-512 batches."""
    from layamd_b200.synthetic import workloads
    g = np.load(os.path.join(GOLD, case + ".npz"))
    lens, ids, nmark, markers, qtypes = workloads.flatten(getattr(workloads, workload)(synth.ARCHS[arch]))
    assert len(lens) == B
    assert (lens == g["lens"]).all() and (nmark == g["nmark"]).all() and (qtypes == g["qtypes"]).all()
    assert (markers == g["markers"]).all() and int(ids.astype(np.int64).sum()) == int(g["ids_sum"])
    assert g["logits"].shape == (int(nmark.sum()),) and g["act"].shape == (B, 2)
    assert np.isfinite(g["logits"]).all() and np.isfinite(g["act"]).all()


@pytest.mark.slow
def test_oracle_on_c2_questions_matches_reference_batch():
    """Three C2 questions (shortest, median, longest) through the oracle against the reference's
    batched C2 logits: padding inside the reference's length-sorted batches does not change them."""
    from layamd_b200.synthetic import workloads
    ck = synth.checkpoint("large", 0)
    w = synth.load_weights(ck)
    check_fingerprint(w, "large_weights_fp.npz")
    o = om.Oracle(w, synth.load_arch(ck))
    qs = workloads.c2(synth.ARCHS["large"], seed=1)
    g = np.load(os.path.join(GOLD, "large_c2_logits.npz"))
    offs = np.concatenate([[0], np.cumsum(g["nmark"])])
    order = sorted(range(len(qs)), key=lambda i: len(qs[i]["ids"]))
    for i in (order[0], order[len(order) // 2], order[-1]):
        lo, ac = o.forward_one(qs[i]["ids"], qs[i]["markers"], qs[i]["qtype"])
        assert np.abs(lo - g["logits"][offs[i]:offs[i + 1]]).max() < 2e-5
        assert np.abs(ac - g["act"][i]).max() < 2e-5 * max(1.0, np.abs(g["act"][i]).max())
