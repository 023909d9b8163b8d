"""Throughput and latency of the engine on the other benchmark configurations (C3, C4), one JSON line.

  python -m layamd_b200.workload_bench --workload c3 [--devices 0,1,...,7]
  python -m layamd_b200.workload_bench --workload c4 [--devices ...] [--calls 50] [--batch1-calls 200]

C3: mmBERT-base architecture (22 layers, d768, 12 heads, GeGLU 1152, vocab 256000, max_len 1024),
    B=128 sequences with L ~ U[64,1024], one 3-option choice question each.
C4: ModernBERT-large architecture at max_len 1024, B=256 sequences with L log-uniform in [128,1024],
    question types cycling choice / score / yes-no with 2-6 options.
Weights are the seeded random-init checkpoints (N(0,0.02), seed 0) served in bf16; inputs are the
seeded synthetic batches of layamd_b200/synthetic/workloads.py. One handle over the listed GPUs shards every call's
questions across them (no collective).

Reported: `value` decisions/s with the packed inputs resident in HBM (laya_stage + laya_replay: CUDA
events on the engine streams, slowest device), `e2e` decisions/s of laya_forward_batch calls from
host arrays (wall clock), per-call p50/p99 latency of full-batch calls, and for C4 the batch-1 p50 /
p99 at L=512 (the C1 shape).
"""
import argparse
import ctypes
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

from layamd_b200.synthetic import synth, workloads  # noqa: E402  (checkpoint generator and input batches only)
from layamd_b200 import load_lib  # noqa: E402

CONFIGS = {
    "c3": ("base", workloads.c3, "C3: mmBERT-base (22 layers, d768, GeGLU 1152, vocab 256000), B=128, "
                                 "L~U[64,1024] (seed 3), one 3-option choice question per sequence"),
    "c4": ("large1024", workloads.c4, "C4: ModernBERT-large at max_len 1024, B=256, L log-uniform [128,1024] "
                                      "(seed 4), choice/score/yes-no 1:1:1 with 2-6 options"),
}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--workload", choices=sorted(CONFIGS), default="c4")
    ap.add_argument("--devices", default="0")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--calls", type=int, default=50, help="full-batch calls for the per-call latency")
    ap.add_argument("--batch1-calls", type=int, default=200, help="C1-shape calls for the batch-1 latency (c4)")
    ap.add_argument("--batch", type=int, default=0,
                    help="questions per call (default: the configuration's B); e.g. 8x B over 8 GPUs gives every "
                         "GPU about one configuration's load through one handle")
    args = ap.parse_args(argv)
    arch_name, gen, desc = CONFIGS[args.workload]
    arch = synth.ARCHS[arch_name]
    ck = synth.checkpoint(arch_name, 0)
    qs = gen(arch, B=args.batch) if args.batch > 0 else gen(arch)
    if args.batch > 0:
        desc += "; B=%d questions per call" % args.batch
    lens, ids, nmark, markers, qtypes = workloads.flatten(qs)
    # one pass per replica: the replica's share of the rows (longest-first assignment keeps every
    # replica within about one question of the mean) with room to spare
    ndev_req = len([d for d in args.devices.split(",") if d.strip()])
    per_dev = int(lens.sum()) // max(1, ndev_req) * 5 // 4 + 4096
    os.environ.setdefault("LAYA_MAX_TOKENS", str(max(131072, per_dev)))
    L = load_lib()
    h = L.laya_create_ex(ck.encode(), 0, args.devices.encode())
    if not h:
        raise SystemExit("laya_create_ex failed")
    ndev = L.laya_num_devices(h)
    n_act = L.laya_n_act(h)
    IP, FP = ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_float)
    p = lambda a: a.ctypes.data_as(IP)  # noqa: E731
    lo = np.zeros(int(nmark.sum()), np.float32)
    ac = np.zeros((len(qs), n_act), np.float32)

    def call():
        rc = L.laya_forward_batch(h, len(qs), p(lens), p(ids), p(nmark), p(markers), p(qtypes),
                                  lo.ctypes.data_as(FP), ac.ctypes.data_as(FP))
        assert rc == 0, "laya_forward_batch returned %d" % rc

    # device-resident throughput
    rc = L.laya_stage(h, len(qs), p(lens), p(ids), p(nmark), p(markers), p(qtypes))
    value = None
    if rc == 0:
        ms = ctypes.c_double(0)
        assert L.laya_replay(h, args.warmup, ctypes.byref(ms)) == 0
        assert L.laya_replay(h, args.steps, ctypes.byref(ms)) == 0
        value = len(qs) * args.steps / (ms.value / 1e3)
    # end to end + per-call latency
    for _ in range(args.warmup):
        call()
    ts = []
    for _ in range(max(args.calls, args.steps)):
        t0 = time.perf_counter()
        call()
        ts.append(time.perf_counter() - t0)
    e2e = len(qs) / float(np.mean(ts))
    line = {"workload": desc, "n_gpus": ndev, "decisions_per_call": len(qs), "tokens_per_call": int(lens.sum()),
            "value": value, "unit": "decisions/s", "e2e": e2e,
            "call_p50_ms": 1e3 * float(np.percentile(ts, 50)), "call_p99_ms": 1e3 * float(np.percentile(ts, 99)),
            "calls": len(ts), "dtype": "bf16", "data": "synthetic (seeded random-init weights and token ids)"}
    if args.workload == "c4" and args.batch1_calls > 0:
        q1 = workloads.c1(arch)
        l1, i1, n1, m1, t1 = workloads.flatten(q1)
        lo1 = np.zeros(3, np.float32)
        ac1 = np.zeros((1, n_act), np.float32)
        for _ in range(10):
            L.laya_forward_batch(h, 1, p(l1), p(i1), p(n1), p(m1), p(t1), lo1.ctypes.data_as(FP), ac1.ctypes.data_as(FP))
        tb = []
        for _ in range(args.batch1_calls):
            t0 = time.perf_counter()
            L.laya_forward_batch(h, 1, p(l1), p(i1), p(n1), p(m1), p(t1), lo1.ctypes.data_as(FP), ac1.ctypes.data_as(FP))
            tb.append(time.perf_counter() - t0)
        line["batch1_p50_ms"] = 1e3 * float(np.percentile(tb, 50))
        line["batch1_p99_ms"] = 1e3 * float(np.percentile(tb, 99))
        line["batch1_calls"] = len(tb)
    print(json.dumps(line), flush=True)
    L.laya_destroy(h)
    return 0


if __name__ == "__main__":
    sys.exit(main())
