"""Host-side multi-rank logic on CPU (gloo, world size 2): the barrier and max-over-ranks timing
reduction bench.py uses under torchrun, and the request-sharding rule of the engine (longest modelled
device time first onto the least-loaded replica, input order kept inside each shard), restated and
checked for balance."""
import os
import socket
import subprocess
import sys
import textwrap

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_bench_dist_max_and_barrier_two_ranks(tmp_path):
    script = tmp_path / "worker.py"
    script.write_text(textwrap.dedent("""
        import os, sys
        sys.path.insert(0, %r)
        import bench
        d = bench.Dist(int(os.environ["WORLD_SIZE"]))
        r = int(os.environ["RANK"])
        d.barrier()
        m = d.max(10.0 + r * 5.0)
        d.barrier()
        print("RESULT", r, m, flush=True)
        d.close()
    """ % ROOT))
    port = free_port()
    procs = []
    for r in range(2):
        env = dict(os.environ, RANK=str(r), LOCAL_RANK=str(r), WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                   MASTER_PORT=str(port))
        procs.append(subprocess.Popen([sys.executable, str(script)], env=env, stdout=subprocess.PIPE,
                                      stderr=subprocess.STDOUT, text=True))
    outs = [p.communicate(timeout=240)[0] for p in procs]
    for p, o in zip(procs, outs):
        assert p.returncode == 0, o
    vals = sorted(float(line.split()[2]) for o in outs for line in o.splitlines() if line.startswith("RESULT"))
    assert vals == [15.0, 15.0]


# ModernBERT-large (hidden 1024, GeGLU 2624, 28 layers, 10 global, window 128) and mmBERT-base
MODELS = {"large": (1024, 2624, 28, 10, 128), "mmbert": (768, 1152, 22, 8, 128)}


def question_cost(L, k, d, inter, nl, ng, window):
    """Modelled device time of one question (quarter-FLOPs at the GEMM rate): algorithmic FLOPs of
    the pass, GEMM FLOPs x4, global / head attention x14, sliding attention x26 (measured B200
    rates 1116 / 316 / 175 TFLOP/s). Sliding keys counted by brute force over the queries."""
    D, I, FF, ns, h = d, inter, 4 * d, nl - ng, window // 2
    band = sum(min(L - 1, q + h) - max(0, q - h) + 1 for q in range(L))
    gemm = (2 * L * (4 * D * D + 3 * I * D) * nl + 2 * L * (4 * D * D + 2 * D * FF) + 2 * L * 3 * D * D
            + 2 * (k + 1) * (D * D + 2 * D * FF) + 2 * k * D * D)
    glob = 4 * D * L * L * (ng + 1) + 4 * D * L * (k + 1)
    return 4 * gemm + 14 * glob + 26 * 4 * D * ns * band


def shard_reference(lens, nmark, G, model):
    """Longest modelled time first onto the least-loaded replica; shards keep input order."""
    cost = [question_cost(L, k, *model) for L, k in zip(lens, nmark)]
    order = sorted(range(len(lens)), key=lambda b: -cost[b])  # stable: ties keep input order
    load = [0] * G
    owner = [0] * len(lens)
    for b in order:
        g = min(range(G), key=lambda i: (load[i], i))
        owner[b] = g
        load[g] += cost[b]
    return [[b for b in range(len(lens)) if owner[b] == g] for g in range(G)], load, cost


def _plan(L, G, lens, nmark, model):
    import ctypes
    IP = ctypes.POINTER(ctypes.c_int)
    la = np.asarray(lens, np.int32)
    nm = np.asarray(nmark, np.int32)
    owner = np.full(len(lens), -1, np.int32)
    assert L.laya_shard_plan(G, len(lens), la.ctypes.data_as(IP), nm.ctypes.data_as(IP), *model,
                             owner.ctypes.data_as(IP)) == 0
    return [[b for b in range(len(lens)) if owner[b] == g] for g in range(G)]


def test_lpt_sharding_is_the_restated_rule_and_balanced():
    from layamd_b200 import load_lib
    L = load_lib()
    rng = np.random.default_rng(0)
    cases = [
        ("large", rng.integers(32, 513, 192).tolist(), rng.integers(2, 6, 192).tolist()),  # C2-like
        ("large", np.round(np.exp(rng.uniform(np.log(128), np.log(1024), 256))).astype(int).tolist(),
         rng.integers(2, 7, 256).tolist()),  # C4-like
        ("mmbert", rng.integers(64, 1025, 128).tolist(), [3] * 128),  # C3-like
        ("large", [1, 1, 2, 1000, 7, 1000, 512, 3], [1, 255, 1, 3, 200, 3, 2, 1]),  # ragged, ties
    ]
    for name, lens, nmark in cases:
        model = MODELS[name]
        for G in (1, 2, 3, 4, 8):
            shards, load, cost = shard_reference(lens, nmark, G, model)
            assert _plan(L, G, lens, nmark, model) == shards  # the engine's rule is the restated one
            assert sorted(b for s in shards for b in s) == list(range(len(lens)))
            assert all(s == sorted(s) for s in shards)
            # LPT bound: the heaviest replica carries at most the mean plus one question
            assert max(load) <= sum(load) / G + max(cost)


def test_cost_model_weights_long_sequences_superlinearly():
    """At context 1024 the global-attention term makes a 1024-token question cost more than two
    512-token ones, which the old length-only rule could not see."""
    m = MODELS["large"]
    c512, c1024 = question_cost(512, 3, *m), question_cost(1024, 3, *m)
    assert c1024 > 2 * c512
    # more options cost more (gathered rows of the last head layer and the scorer)
    assert question_cost(512, 200, *m) > question_cost(512, 2, *m)


def test_shard_plan_rejects_bad_arguments():
    import ctypes
    from layamd_b200 import load_lib
    L = load_lib()
    IP = ctypes.POINTER(ctypes.c_int)
    la = np.asarray([5, 6], np.int32)
    nm = np.asarray([1, 2], np.int32)
    ow = np.zeros(2, np.int32)
    p = lambda a: a.ctypes.data_as(IP)  # noqa: E731
    assert L.laya_shard_plan(0, 2, p(la), p(nm), 1024, 2624, 28, 10, 128, p(ow)) == -1
    assert L.laya_shard_plan(2, 2, p(la), None, 1024, 2624, 28, 10, 128, p(ow)) == -1
    assert L.laya_shard_plan(2, 2, p(la), p(nm), 1024, 2624, 28, 29, 128, p(ow)) == -1
