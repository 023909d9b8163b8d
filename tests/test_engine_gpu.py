"""End-to-end parity of the engine (liblaya_b200.so, through the C ABI) against the golden fixtures
of the reference PyTorch path and against the numpy oracle run on the same seeded inputs.

Tolerances, as the parity contract states them:
  fp32-parity mode  per-layer hidden states max|a-b|/max|b| <= 1e-3; probabilities <= 1e-4 absolute;
                    act logits relative <= 1e-3
  bf16 mode         argmax of every question equal to the oracle's; probability delta < 0.01 and act
                    relative error < 0.05 (the reference's own row tolerance, src/test_parity.cpp:69)
"""
import ctypes
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

from oracle import model as om  # noqa: E402
from layamd_b200.synthetic import synth, workloads  # noqa: E402
from tests.engine_helpers import (Handle, act_rel, argmax_agree, gathered_rows, prob_delta, read_dump,  # noqa: E402
                                  rel)

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ENV = {"LAYA_MAX_TOKENS": 16384}


def questions_of(g):
    qs, io, mo = [], 0, 0
    for L, k, qt in zip(g["lens"], g["nmark"], g["qtypes"]):
        qs.append({"ids": g["ids"][io:io + L].tolist(), "markers": g["markers"][mo:mo + k].tolist(), "qtype": int(qt)})
        io += L
        mo += k
    return qs


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture(scope="module")
def tiny_ckpt():
    return synth.checkpoint("tiny", 0)


@pytest.fixture(scope="module")
def tiny_oracle(tiny_ckpt):
    return om.Oracle(synth.load_weights(tiny_ckpt), synth.load_arch(tiny_ckpt))


@pytest.fixture(scope="module")
def tiny_fp32(tiny_ckpt):
    h = Handle(tiny_ckpt, 1, env=ENV)
    yield h
    h.close()


@pytest.fixture(scope="module")
def tiny_bf16(tiny_ckpt):
    h = Handle(tiny_ckpt, 0, env=ENV)
    yield h
    h.close()


@pytest.fixture(scope="module")
def large_ckpt():
    return synth.checkpoint("large", 0)


@pytest.fixture(scope="module")
def large_oracle(large_ckpt):
    return om.Oracle(synth.load_weights(large_ckpt), synth.load_arch(large_ckpt))


@pytest.fixture(scope="module")
def large_fp32(large_ckpt):
    h = Handle(large_ckpt, 1, env=ENV)
    yield h
    h.close()


@pytest.fixture(scope="module")
def large_bf16(large_ckpt):
    h = Handle(large_ckpt, 0, env={"LAYA_MAX_TOKENS": 65536})
    yield h
    h.close()


@pytest.mark.parametrize("case", ["tiny_mixed", "tiny_k1", "tiny_full"])
def test_tiny_fp32_parity_layers_vs_golden(tiny_fp32, case):
    g = np.load(os.path.join(GOLD, case + ".npz"))
    qs = questions_of(g)
    lo, ac, d = tiny_fp32.forward_dump(qs)
    D = 128
    for key in ["emb"] + ["enc%d" % i for i in range(4)] + ["head0"]:
        assert rel(read_dump(d, key, D), g["t_" + key]) <= 1e-3, key
    # last head layer: the engine keeps only marker rows then CLS rows
    lens = g["lens"]
    offs = np.concatenate([[0], np.cumsum(lens)])
    h1 = g["t_head1"]
    ref = np.concatenate([h1[offs[i] + np.asarray(q["markers"])] for i, q in enumerate(qs)] +
                         [h1[offs[i]:offs[i] + 1] for i in range(len(qs))])
    assert rel(read_dump(d, "head1", D), ref) <= 1e-3
    assert prob_delta(lo, g["logits"], qs) <= 1e-4
    assert act_rel(ac, g["act"]) <= 1e-3


@pytest.mark.parametrize("case", ["tiny_mixed", "tiny_k1", "tiny_full"])
def test_tiny_bf16_vs_golden(tiny_bf16, case):
    g = np.load(os.path.join(GOLD, case + ".npz"))
    qs = questions_of(g)
    rc, lo, ac = tiny_bf16.forward(qs)
    assert rc == 0
    assert argmax_agree(lo, g["logits"], qs)
    assert prob_delta(lo, g["logits"], qs) < 0.01
    assert act_rel(ac, g["act"]) < 0.05


def test_tiny_random_batches_vs_oracle(tiny_fp32, tiny_bf16, tiny_oracle):
    a = synth.ARCHS["tiny"]
    for seed in range(3):
        qs = workloads.mixed(a, 40, seed=100 + seed, kmax=12)
        lo_o, ac_o, _ = tiny_oracle.forward_batch(qs)
        rc, lo, ac = tiny_fp32.forward(qs)
        assert rc == 0
        assert prob_delta(lo, lo_o, qs) <= 1e-4
        assert act_rel(ac, ac_o) <= 1e-3
        rc, lo, ac = tiny_bf16.forward(qs)
        assert rc == 0
        assert prob_delta(lo, lo_o, qs) < 0.01
        assert act_rel(ac, ac_o) < 0.05


def test_large_c1_fp32_parity_per_layer(large_fp32, large_oracle):
    a = synth.ARCHS["large"]
    qs = workloads.c1(a)
    lo, ac, d = large_fp32.forward_dump(qs)
    lo_o, ac_o, caps = large_oracle.forward_batch(qs, capture=True)
    D = a.d
    worst = {}
    for key in ["emb"] + ["enc%d" % i for i in range(a.layers)] + ["final", "head0"]:
        worst[key] = rel(read_dump(d, key, D), caps[0][key])
    worst["head1"] = rel(read_dump(d, "head1", D), gathered_rows("head1", qs, caps))
    bad = {k: v for k, v in worst.items() if v > 1e-3}
    assert not bad, bad
    assert prob_delta(lo, lo_o, qs) <= 1e-4
    assert act_rel(ac, ac_o) <= 1e-3
    # and against the reference's own golden C1 logits
    g = np.load(os.path.join(GOLD, "large_c1.npz"))
    assert prob_delta(lo, g["logits"], qs) <= 1e-4


def test_large_c1_bf16(large_bf16, large_oracle):
    qs = workloads.c1(synth.ARCHS["large"])
    rc, lo, ac = large_bf16.forward(qs)
    assert rc == 0
    lo_o, ac_o, _ = large_oracle.forward_batch(qs)
    assert argmax_agree(lo, lo_o, qs)
    assert prob_delta(lo, lo_o, qs) < 0.01
    assert act_rel(ac, ac_o) < 0.05


def test_large_c2_bf16_all_192_vs_reference(large_bf16):
    """The benchmark's own batch, every question: C2 (64 states x 3 questions, 52,287 tokens) through
    one laya_forward_batch call in bf16, against the reference PyTorch path's fp32 logits for the same
    192 questions (tests/golden/large_c2_logits.npz, made by make_golden.py --c2)."""
    qs = workloads.c2(synth.ARCHS["large"])
    g = np.load(os.path.join(GOLD, "large_c2_logits.npz"))
    lens, ids, nmark, markers, qtypes = workloads.flatten(qs)
    assert (lens == g["lens"]).all() and (nmark == g["nmark"]).all() and (markers == g["markers"]).all()
    assert int(ids.astype(np.int64).sum()) == int(g["ids_sum"])
    rc, lo, ac = large_bf16.forward(qs)
    assert rc == 0 and np.isfinite(lo).all() and np.isfinite(ac).all()
    assert len(qs) == 192
    assert prob_delta(lo, g["logits"], qs) < 0.01
    assert act_rel(ac, g["act"]) < 0.05
    assert argmax_agree(lo, g["logits"], qs)


def test_seq512_batch_bf16_vs_reference(large_bf16):
    """The bench's fixed-length batch (128 choice questions of exactly 512 tokens, 3 options each)
    in one bf16 call, against the reference's logits for it (tests/golden/large_seq512_logits.npz,
    made by make_golden.py --seq512)."""
    qs = workloads.seq512(synth.ARCHS["large"])
    g = np.load(os.path.join(GOLD, "large_seq512_logits.npz"))
    lens, ids, nmark, markers, qtypes = workloads.flatten(qs)
    assert (lens == g["lens"]).all() and (markers == g["markers"]).all()
    assert int(ids.astype(np.int64).sum()) == int(g["ids_sum"])
    rc, lo, ac = large_bf16.forward(qs)
    assert rc == 0
    assert prob_delta(lo, g["logits"], qs) < 0.01
    assert act_rel(ac, g["act"]) < 0.05
    assert argmax_agree(lo, g["logits"], qs)


def test_large_c2_fp32_parity_all_192_vs_reference(large_fp32):
    """The same 192 questions in fp32-parity mode, at the parity contract's tolerance, through an
    engine whose 16,384-row passes split the 52,287-token batch into several passes."""
    qs = workloads.c2(synth.ARCHS["large"])
    g = np.load(os.path.join(GOLD, "large_c2_logits.npz"))
    rc, lo, ac = large_fp32.forward(qs)
    assert rc == 0
    assert prob_delta(lo, g["logits"], qs) <= 1e-4
    assert act_rel(ac, g["act"]) <= 1e-3
    assert argmax_agree(lo, g["logits"], qs)


def test_validation_contract(tiny_bf16):
    a = synth.ARCHS["tiny"]
    good = workloads.mixed(a, 3, seed=7, kmax=3)
    bad_cases = [
        [dict(good[0], ids=[])],                                              # len 0
        [dict(good[0], ids=good[0]["ids"] + [5] * (a.max_len + 1))],          # len > max_len
        [dict(good[1], markers=[])],                                          # nmark 0
        [dict(good[1], markers=[len(good[1]["ids"])])],                       # marker == len
        [dict(good[1], markers=[-1])],                                        # marker < 0
        [dict(good[2], ids=[5] * 120, markers=[1] * 256)],                    # 256 markers
        [dict(good[0], ids=[a.vocab] + good[0]["ids"][1:])],                  # id past the vocabulary
        [dict(good[0], ids=[-1] + good[0]["ids"][1:])],                       # negative id
        [good[0], dict(good[1], qtype=3)],                                    # unknown question type
    ]
    for qs in bad_cases:
        rc, lo, ac = tiny_bf16.forward(qs)
        assert rc == -1
        assert np.isnan(ac).all()  # outputs untouched
    # an empty batch is a successful no-op (the reference's loops simply do not run,
    # src/engine.hip:491-497), and the next call is unaffected
    one = np.zeros(1, np.int32)
    lo0 = np.full(1, np.nan, np.float32)
    ac0 = np.full((1, tiny_bf16.n_act), np.nan, np.float32)
    IPt, FPt = ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_float)
    assert tiny_bf16.L.laya_forward_batch(tiny_bf16.h, 0, *[one.ctypes.data_as(IPt)] * 5,
                                          lo0.ctypes.data_as(FPt), ac0.ctypes.data_as(FPt)) == 0
    assert np.isnan(lo0).all() and np.isnan(ac0).all()
    rc, lo, ac = tiny_bf16.forward(good)
    assert rc == 0 and np.isfinite(lo).all() and np.isfinite(ac).all()


def test_255_markers_and_one_token(tiny_fp32, tiny_oracle):
    a = synth.ARCHS["tiny"]
    rng = np.random.default_rng(5)
    # tiny max_len is 128, so 127 markers is the most a question can hold here; the large model
    # case below covers 255
    q1 = {"ids": rng.integers(5, a.vocab, 128).tolist(), "markers": list(range(1, 128)), "qtype": 0}
    q2 = {"ids": [a.cls_id], "markers": [0], "qtype": 2}
    qs = [q1, q2, workloads.mixed(a, 1, seed=9)[0]]
    rc, lo, ac = tiny_fp32.forward(qs)
    assert rc == 0
    lo_o, ac_o, _ = tiny_oracle.forward_batch(qs)
    assert prob_delta(lo, lo_o, qs) <= 1e-4
    assert act_rel(ac, ac_o) <= 1e-3


def test_large_255_markers(large_bf16, large_oracle):
    a = synth.ARCHS["large"]
    rng = np.random.default_rng(6)
    q = {"ids": rng.integers(5, a.vocab, 400).tolist(), "markers": sorted(rng.choice(np.arange(1, 400), 255, replace=False).tolist()),
         "qtype": 0}
    rc, lo, ac = large_bf16.forward([q])
    assert rc == 0
    lo_o, ac_o, _ = large_oracle.forward_batch([q])
    assert prob_delta(lo, lo_o, [q]) < 0.01
    assert act_rel(ac, ac_o) < 0.05


def test_multipass_equals_single_pass(tiny_ckpt):
    """Packing invariance: the same questions cut into many small passes give the single pass's
    results. The attention kernel is pinned (LAYA_ATTN_SMALL=0), since small passes would otherwise
    take the mma.sync attention, whose bf16 rounding differs (checked separately)."""
    a = synth.ARCHS["tiny"]
    qs = workloads.mixed(a, 60, seed=11, kmax=8)
    one = Handle(tiny_ckpt, 0, env={"LAYA_MAX_TOKENS": 16384, "LAYA_ATTN_SMALL": 0})
    many = Handle(tiny_ckpt, 0, env={"LAYA_MAX_TOKENS": 16384, "LAYA_PASS_TOKENS": 300, "LAYA_MAX_SEQS": 5,
                                     "LAYA_ATTN_SMALL": 0})
    try:
        rc1, lo1, ac1 = one.forward(qs)
        rc2, lo2, ac2 = many.forward(qs)
        assert rc1 == 0 and rc2 == 0
        assert rel(lo2, lo1) < 1e-5 and rel(ac2, ac1) < 1e-5
    finally:
        one.close()
        many.close()


def test_small_pass_attention_choice_matches_tcgen05_path(large_ckpt, large_oracle):
    """Passes of at most 1024 rows run the sliding-window layers (and at 512 rows the global ones) on
    the mma.sync attention kernel. At batch 1 (C1 shape, 512 rows) its results agree with the tcgen05
    path and with the oracle at the bf16 tolerance (probability delta < 0.01, act < 0.05)."""
    qs = workloads.c1(synth.ARCHS["large"])
    small = Handle(large_ckpt, 0, env={"LAYA_MAX_TOKENS": 4096})
    tc = Handle(large_ckpt, 0, env={"LAYA_MAX_TOKENS": 4096, "LAYA_ATTN_SMALL": 0})
    try:
        r1, r2 = small.forward(qs), tc.forward(qs)
    finally:
        small.close()
        tc.close()
    assert r1[0] == 0 and r2[0] == 0
    assert not np.array_equal(r1[1], r2[1])  # the two kernels really ran
    lo_o, ac_o, _ = large_oracle.forward_batch(qs)
    for lo, ac in ((r1[1], r1[2]), (r2[1], r2[2])):
        assert prob_delta(lo, lo_o, qs) < 0.01 and act_rel(ac, ac_o) < 0.05
    assert prob_delta(r1[1], r2[1], qs) < 0.01


def test_graph_replay_is_bitwise_stable(tiny_ckpt):
    a = synth.ARCHS["tiny"]
    qs = workloads.mixed(a, 20, seed=12)
    g = Handle(tiny_ckpt, 0, env={"LAYA_MAX_TOKENS": 16384})
    e = Handle(tiny_ckpt, 0, env={"LAYA_MAX_TOKENS": 16384, "LAYA_GRAPHS": 0})
    try:
        r1 = g.forward(qs)   # captures the graph
        r2 = g.forward(qs)   # replays it
        r3 = e.forward(qs)   # eager launches
        for r in (r1, r2, r3):
            assert r[0] == 0
        assert np.array_equal(r1[1], r2[1]) and np.array_equal(r1[2], r2[2])
        assert np.array_equal(r1[1], r3[1]) and np.array_equal(r1[2], r3[2])
    finally:
        g.close()
        e.close()


def test_order_invariance_full_c2(large_bf16):
    """Size-independent property at the benchmark's full size: a question's outputs do not depend on
    where it sits in the batch (no cross-sequence attention, no row coupling in the GEMMs)."""
    qs = workloads.c2(synth.ARCHS["large"])
    rc, lo, ac = large_bf16.forward(qs)
    assert rc == 0
    perm = np.random.default_rng(0).permutation(len(qs))
    rc, lo_p, ac_p = large_bf16.forward([qs[i] for i in perm])
    assert rc == 0
    per = []
    o = 0
    for q in qs:
        per.append(lo[o:o + len(q["markers"])])
        o += len(q["markers"])
    per_p = [per[i] for i in perm]
    assert rel(lo_p, np.concatenate(per_p)) < 1e-5
    assert rel(ac_p, ac[perm]) < 1e-5


def test_pair_tile_matches_single_cta_tiles(large_ckpt, large_bf16):
    """At C2 size the engine runs its GEMMs on the CTA-pair 256 x 256 tile; the single-CTA tiles
    (LAYA_NO_PAIR_GEMM) must give the same decisions."""
    qs = workloads.c2(synth.ARCHS["large"], states=16)
    rc, lo, ac = large_bf16.forward(qs)
    assert rc == 0
    h = Handle(large_ckpt, 0, env={"LAYA_MAX_TOKENS": 65536, "LAYA_NO_PAIR_GEMM": 1})
    try:
        rc2, lo2, ac2 = h.forward(qs)
    finally:
        h.close()
    assert rc2 == 0
    assert prob_delta(lo, lo2, qs) < 1e-3
    assert act_rel(ac, ac2) < 1e-2


def test_splitk_engine_matches_whole_k(large_ckpt, large_bf16):
    """With LAYA_SPLITK=1 a batch-1 pass (512 rows: too few 128 x 128 tiles to fill the GPU) runs its
    GEMMs with the K loop split across CTAs; the decisions equal the whole-K ones."""
    qs = workloads.c2(synth.ARCHS["large"], states=1)
    rc, lo, ac = large_bf16.forward(qs)
    assert rc == 0
    h = Handle(large_ckpt, 0, env={"LAYA_MAX_TOKENS": 4096, "LAYA_SPLITK": 1})
    try:
        rc2, lo2, ac2 = h.forward(qs)
        rc3, lo3, ac3 = h.forward(qs)
    finally:
        h.close()
    assert rc2 == 0 and rc3 == 0
    assert prob_delta(lo, lo2, qs) < 1e-3
    assert act_rel(ac, ac2) < 1e-2
    # slices are summed in a fixed order: a repeated call is bitwise identical
    assert np.array_equal(lo2, lo3) and np.array_equal(ac2, ac3)


def _device_list():
    """Every GPU of the box, or two replicas on GPU 0 when there is only one (each replica has its own
    weights, arena, stream and graphs, so the sharded path runs the same way)."""
    n = torch.cuda.device_count()
    return ",".join(str(i) for i in range(n)) if n >= 2 else "0,0"


def test_multi_device_sharding_matches_one_device(tiny_ckpt):
    """One handle over several replicas (LAYA_DEVICES-style device list) shards each call's questions;
    every question's outputs equal the single-replica ones."""
    qs = workloads.mixed(synth.ARCHS["tiny"], 50, seed=13, kmax=6)
    devs = _device_list()
    one = Handle(tiny_ckpt, 1, devices="0", env=ENV)
    many = Handle(tiny_ckpt, 1, devices=devs, env=ENV)
    try:
        assert many.L.laya_num_devices(many.h) == len(devs.split(","))
        r1 = one.forward(qs)
        for _ in range(2):  # the replicas' workers are reused by the second call
            r2 = many.forward(qs)
            assert r1[0] == 0 and r2[0] == 0
            assert rel(r2[1], r1[1]) < 1e-5 and rel(r2[2], r1[2]) < 1e-5
    finally:
        one.close()
        many.close()


def test_replica_failure_is_reported_and_the_next_call_succeeds(tiny_ckpt):
    """Host-side failure injection (LAYA_FAIL_REPLICA=1): replica 1 returns an error for its next shard
    before uploading or launching anything. The sharded call returns -2 only after every replica has
    finished its part; the next call on the same handle runs every replica and matches one device."""
    qs = workloads.mixed(synth.ARCHS["tiny"], 40, seed=21, kmax=5)
    devs = _device_list()
    one = Handle(tiny_ckpt, 0, devices="0", env=ENV)
    many = Handle(tiny_ckpt, 0, devices=devs, env=dict(ENV, LAYA_FAIL_REPLICA="1:1"))
    try:
        rc, lo, ac = many.forward(qs)
        assert rc == -2
        # the replicas that did run wrote their shards: some questions have results, others not
        assert np.isfinite(ac).any() and np.isnan(ac).any()
        r1 = one.forward(qs)
        r2 = many.forward(qs)
        assert r1[0] == 0 and r2[0] == 0
        assert np.isfinite(r2[2]).all()
        assert rel(r2[1], r1[1]) < 1e-5 and rel(r2[2], r1[2]) < 1e-5
    finally:
        one.close()
        many.close()


def test_stage_replay_matches_forward(large_bf16):
    from tests.engine_helpers import FP, IP
    qs = workloads.c2(synth.ARCHS["large"], states=8)
    rc, lo, ac = large_bf16.forward(qs)
    assert rc == 0
    L = large_bf16.L
    lens, ids, nmark, markers, qtypes = workloads.flatten(qs)
    p = lambda x: x.ctypes.data_as(IP)  # noqa: E731
    assert L.laya_stage(large_bf16.h, len(qs), p(lens), p(ids), p(nmark), p(markers), p(qtypes)) == 0
    import ctypes
    ms = ctypes.c_double(0)
    assert L.laya_replay(large_bf16.h, 3, ctypes.byref(ms)) == 0
    assert ms.value > 0
    lo2 = np.zeros_like(lo)
    ac2 = np.zeros_like(ac)
    assert L.laya_staged_results(large_bf16.h, lo2.ctypes.data_as(FP), ac2.ctypes.data_as(FP)) == 0
    assert rel(lo2, lo) < 1e-5 and rel(ac2, ac) < 1e-5
    # the profiled copy of the staged graph: the same results, and one timed entry per stage per pass
    # (the last replay's)
    L.laya_prof_reset(large_bf16.h)
    assert L.laya_replay_profiled(large_bf16.h, 2) == 0
    lo3 = np.zeros_like(lo)
    ac3 = np.zeros_like(ac)
    assert L.laya_staged_results(large_bf16.h, lo3.ctypes.data_as(FP), ac3.ctypes.data_as(FP)) == 0
    assert np.array_equal(lo3, lo2) and np.array_equal(ac3, ac2)
    for name in (b"gemm_qkv", b"gemm_mlp_in", b"attn_global", b"attn_sliding"):
        t, n = ctypes.c_double(0), ctypes.c_longlong(0)
        assert L.laya_prof_get(large_bf16.h, name, ctypes.byref(t), ctypes.byref(n)) == 0
        assert t.value > 0
    t, n = ctypes.c_double(0), ctypes.c_longlong(0)
    L.laya_prof_get(large_bf16.h, b"gemm_qkv", ctypes.byref(t), ctypes.byref(n))
    assert n.value == synth.ARCHS["large"].layers
    L.laya_prof_reset(large_bf16.h)


def test_split_k_layernorm_fusion_is_exact(large_ckpt, large_bf16):
    """At 512 rows the attention-out and MLP-out GEMMs run split-K, and their reduce kernels also write
    the LayerNorm that follows (the MLP norm, the next layer's attention norm). With that fusion off
    (LAYA_SPLIT_LN=0: the same K splits) the LayerNorm kernel computes the same rows from the same x
    with the same arithmetic: the same bits out."""
    qs = workloads.c1(synth.ARCHS["large"])
    rc, lo, ac = large_bf16.forward(qs)
    assert rc == 0
    h = Handle(large_ckpt, 0, env={"LAYA_MAX_TOKENS": 65536, "LAYA_SPLIT_LN": 0})
    try:
        rc2, lo2, ac2 = h.forward(qs)
    finally:
        h.close()
    assert rc2 == 0
    assert np.array_equal(lo, lo2) and np.array_equal(ac, ac2)
