"""Parity at the other two benchmark configurations, against the oracle on the same seeded
checkpoints: mmBERT-base (C3: d 768, 12 heads, 22 layers, GeGLU 1152, vocabulary 256000, pad id 0,
context 1024) and ModernBERT-large at context 1024 (C4: sequences past 512 tokens, RoPE positions
and global attention up to 1024 keys), in fp32-parity and bf16 mode."""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from layamd_b200.synthetic import synth, workloads  # noqa: E402
from oracle import model as om  # noqa: E402
from tests.engine_helpers import Handle, act_rel, argmax_agree, gathered_rows, prob_delta, read_dump, rel  # noqa: E402

pytestmark = pytest.mark.gpu
ENV = {"LAYA_MAX_TOKENS": 16384}
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def spread(qs, n):
    """n questions spread over the batch's lengths, the longest included."""
    order = sorted(range(len(qs)), key=lambda i: len(qs[i]["ids"]))
    picks = sorted({order[int(round(j * (len(order) - 1) / (n - 1)))] for j in range(n)})
    return [qs[i] for i in picks]


def check_both_modes(ckpt, qs, oracle):
    lo_o, ac_o, _ = oracle.forward_batch(qs)
    for precision, dp, da in ((1, 1e-4, 1e-3), (0, 0.01, 0.05)):
        h = Handle(ckpt, precision, env=ENV)
        try:
            rc, lo, ac = h.forward(qs)
        finally:
            h.close()
        assert rc == 0
        assert prob_delta(lo, lo_o, qs) <= dp, precision
        assert act_rel(ac, ac_o) <= da, precision
        if precision == 0:
            assert argmax_agree(lo, lo_o, qs)


def test_mmbert_base_c3_shapes():
    ck = synth.checkpoint("base", 0)
    o = om.Oracle(synth.load_weights(ck), synth.load_arch(ck))
    qs = spread(workloads.c3(synth.ARCHS["base"]), 6)
    assert max(len(q["ids"]) for q in qs) > 900
    check_both_modes(ck, qs, o)


def test_large_context_1024_c4_shapes():
    ck = synth.checkpoint("large1024", 0)
    a = synth.load_arch(ck)
    o = om.Oracle(synth.load_weights(ck), a)
    qs = spread(workloads.c4(synth.ARCHS["large1024"]), 6)
    assert max(len(q["ids"]) for q in qs) > 1000
    check_both_modes(ck, qs, o)
    # every hidden state of the longest question in fp32-parity mode (max |a - b| / max |b| <= 1e-3)
    q = [max(qs, key=lambda x: len(x["ids"]))]
    h = Handle(ck, 1, env=ENV)
    try:
        lo, ac, d = h.forward_dump(q)
    finally:
        h.close()
    _, _, caps = o.forward_batch(q, capture=True)
    worst = {k: rel(read_dump(d, k, a.d), caps[0][k])
             for k in ["emb"] + ["enc%d" % i for i in range(a.layers)] + ["final", "head0"]}
    worst["head1"] = rel(read_dump(d, "head1", a.d), gathered_rows("head1", q, caps))
    bad = {k: v for k, v in worst.items() if v > 1e-3}
    assert not bad, bad
    assert np.isfinite(lo).all()


@pytest.mark.parametrize("arch,case", [("base", "base_c3"), ("large1024", "large1024_c4")])
def test_fp32_parity_against_reference_golden(arch, case):
    """The engine in fp32-parity mode against the reference's own outputs at C3 and C4
    (tests/golden/base_c3.npz, large1024_c4.npz: ref/rl_common.py + transformers on the same seeded
    checkpoint): probabilities within 1e-4, act logits within 1e-3, and per layer the row norms of
    every packed row and the full sampled rows of the first (longest) question within
    max|a-b|/max|b| <= 1e-3."""
    ck = synth.checkpoint(arch, 0)
    a = synth.load_arch(ck)
    g = np.load(os.path.join(GOLD, case + ".npz"))
    qs, io, mo = [], 0, 0
    for L, k, qt in zip(g["lens"], g["nmark"], g["qtypes"]):
        qs.append({"ids": g["ids"][io:io + L].tolist(), "markers": g["markers"][mo:mo + k].tolist(), "qtype": int(qt)})
        io += L
        mo += k
    h = Handle(ck, 1, env=ENV)
    try:
        lo, ac, d = h.forward_dump(qs)
    finally:
        h.close()
    assert prob_delta(lo, g["logits"], qs) <= 1e-4
    assert act_rel(ac, g["act"]) <= 1e-3
    lens = [len(q["ids"]) for q in qs]
    T = sum(lens)
    rows = g["sample_rows"]
    worst = {}
    for key in ["emb"] + ["enc%d" % i for i in range(a.layers)] + ["head0"]:
        t = read_dump(d, key, a.d)[:T]
        worst[key] = max(rel(np.linalg.norm(t, axis=-1), g["n_" + key]), rel(t[rows], g["s_" + key]))
    offs = np.cumsum([0] + lens[:-1])
    idx = [int(o + m) for o, q in zip(offs, qs) for m in q["markers"]] + [int(o) for o in offs]
    t = read_dump(d, "head1", a.d)[:len(idx)]  # gathered rows: every question's markers, then its CLS row
    worst["head1"] = rel(np.linalg.norm(t, axis=-1), g["n_head1"][idx])
    bad = {k: v for k, v in worst.items() if v > 1e-3}
    assert not bad, bad


@pytest.mark.parametrize("arch,workload,case", [("base", "c3", "base_c3_logits"),
                                                ("large1024", "c4", "large1024_c4_logits")])
def test_whole_benchmark_batch_against_reference(arch, workload, case):
    """The whole batch workload_bench serves at C3 (128 mmBERT-base questions, L ~ U[64,1024]) and C4
    (256 ModernBERT-large context-1024 questions, L log-uniform in [128,1024]) through one
    laya_forward_batch call, against the reference's logits for the same questions
    (tests/golden/<case>.npz, made by make_golden.py --c3c4): fp32-parity mode at the parity contract's
    tolerance and bf16 at the reference's row tolerance with the argmax rule."""
    ck = synth.checkpoint(arch, 0)
    qs = getattr(workloads, workload)(synth.ARCHS[arch])
    g = np.load(os.path.join(GOLD, case + ".npz"))
    lens, ids, nmark, markers, qtypes = workloads.flatten(qs)
    assert (lens == g["lens"]).all() and (nmark == g["nmark"]).all() and (markers == g["markers"]).all()
    assert int(ids.astype(np.int64).sum()) == int(g["ids_sum"])
    for precision, dp, da in ((1, 1e-4, 1e-3), (0, 0.01, 0.05)):
        h = Handle(ck, precision, env={"LAYA_MAX_TOKENS": 65536})
        try:
            rc, lo, ac = h.forward(qs)
        finally:
            h.close()
        assert rc == 0
        assert prob_delta(lo, g["logits"], qs) <= dp, precision
        assert act_rel(ac, g["act"]) <= da, precision
        assert argmax_agree(lo, g["logits"], qs), precision
