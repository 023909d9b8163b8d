"""Host-side multi-rank logic on CPU (gloo, world size 2): the barrier and max-over-ranks timing
reduction bench.py uses under torchrun, and the request-sharding rule of the engine (longest question
first onto the least-loaded replica, input order kept inside each shard), restated and checked for
balance."""
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


def shard_reference(lens, G):
    """Longest question first onto the least-loaded replica (cost len + 64), shard keeps input order."""
    order = sorted(range(len(lens)), key=lambda b: -lens[b])  # stable for equal lengths
    load = [0] * G
    owner = [0] * len(lens)
    for b in order:
        g = int(np.argmin(load))
        owner[b] = g
        load[g] += lens[b] + 64
    return [[b for b in range(len(lens)) if owner[b] == g] for g in range(G)], load


def test_lpt_sharding_is_balanced():
    import ctypes
    from layamd_b200 import load_lib
    L = load_lib()
    IP = ctypes.POINTER(ctypes.c_int)
    rng = np.random.default_rng(0)
    lens = rng.integers(32, 513, 192).tolist()
    for G in (1, 2, 4, 8):
        shards, load = shard_reference(lens, G)
        la = np.asarray(lens, np.int32)
        owner = np.full(len(lens), -1, np.int32)
        assert L.laya_shard_plan(G, len(lens), la.ctypes.data_as(IP), owner.ctypes.data_as(IP)) == 0
        got = [[b for b in range(len(lens)) if owner[b] == g] for g in range(G)]
        assert got == shards  # the engine's rule is the restated one
        assert sorted(b for s in shards for b in s) == list(range(len(lens)))
        assert all(s == sorted(s) for s in shards)
        # LPT bound: the heaviest replica carries at most the mean plus one question
        assert max(load) <= sum(load) / G + max(lens) + 64
