"""Request-path benchmark: decisions/s and request latency through layamd_b200.server on this engine.

Workload: the C2 shape as requests. 64 states with token lengths L ~ U[32, 512] (random.Random(1)),
each asked three questions (choice with 2-5 options, 3-level score, yes/no) in one request, on the
seeded ModernBERT-large checkpoint with its synthetic word-level tokenizer (one word per token, so
state texts are sized in tokens). Synthetic texts; no dataset.

Measured, one JSON line:
  direct   requests one after another, one engine call each (``Laya.system_one``)
  batched  `clients` threads sending requests back to back for `seconds` through one ``Batcher``
           (decisions/s, request latency p50 / p99, rounds and tokens per round)
  host     prepare + finish alone per request (CPU time of the request path around the engine)
  engine   all 192 questions in one ``forward_batch`` (the engine-only rate for the same inputs)
  many     64 choice questions of 120 options each (300-token states) in one ``forward_batch``: the
           gathered marker rows (7,680) dominate the last head layer and the scorer

    python -m layamd_b200.server_bench [--clients 64] [--seconds 20] [--devices 0,1]
"""
import argparse
import json
import os
import random
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
from layamd_b200 import server as S  # noqa: E402
from layamd_b200.synthetic import synth  # noqa: E402  (seeded checkpoint and tokenizer files only)


def make_requests(n_states=64, seed=1):
    rl = random.Random(seed)
    rng = np.random.default_rng(seed)
    reqs = []
    for i in range(n_states):
        L = rl.randint(32, 512)
        k = rl.randint(2, 5)
        state = " ".join("t%d" % v for v in rng.integers(2000, 40000, max(1, L - 40)))
        questions = {
            "next": {"type": "choice", "instructions": "which action should the agent take next?",
                     "criteria": {"go": "move to the next room", "wait": None, "stop": "stop the task",
                                  "pick": "pick up the key", "drop": None}
                     if k == 5 else ["go", "wait", "stop", "pick"][:k]},
            "quality": {"type": "score", "instructions": "rate the quality of the last step",
                        "criteria": ["bad", "good", "correct and helpful"]},
            "done": {"type": "noul", "instructions": "is the task done?"},
        }
        reqs.append((state, questions))
    return reqs


def pct(xs, q):
    return float(np.percentile(np.asarray(xs) * 1e3, q)) if xs else None


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--arch", default="large")
    ap.add_argument("--clients", type=int, default=64)
    ap.add_argument("--seconds", type=float, default=20.0)
    ap.add_argument("--devices", default="")
    ap.add_argument("--max-tokens", type=int, default=None)
    args = ap.parse_args()

    ck = synth.checkpoint(args.arch, 0)
    t = time.perf_counter()
    lay = S.Laya(ck, devices=args.devices)
    startup = time.perf_counter() - t
    reqs = make_requests()
    nq = sum(len(q) for _, q in reqs)

    # host side alone
    t = time.perf_counter()
    prepared = [lay.prepare(s, q) for s, q in reqs]
    t_prep = (time.perf_counter() - t) / len(reqs)
    fake = [([np.zeros(len(m), np.float32) for _, m, _ in it], np.zeros((len(it), lay.engine.n_act), np.float32))
            for _, _, it in prepared]
    t = time.perf_counter()
    for (qids, qs, it), (lg, ac) in zip(prepared, fake):
        lay.finish(qids, qs, it, lg, ac, 0.0)
    t_fin = (time.perf_counter() - t) / len(reqs)
    tokens = sum(len(s) for _, _, it in prepared for s, _, _ in it)

    # engine only: every question in one call
    items = [x for _, _, it in prepared for x in it]
    seqs, marks, qts = [x[0] for x in items], [x[1] for x in items], [x[2] for x in items]
    for _ in range(2):
        lay.engine.forward_batch(seqs, marks, qts)
    t = time.perf_counter()
    reps = 5
    for _ in range(reps):
        lay.engine.forward_batch(seqs, marks, qts)
    eng_rate = reps * nq / (time.perf_counter() - t)

    # direct requests
    lat = []
    t = time.perf_counter()
    for s, q in reqs:
        t1 = time.perf_counter()
        lay.system_one(s, q)
        lat.append(time.perf_counter() - t1)
    direct_rate = nq / (time.perf_counter() - t)

    # batched requests from concurrent clients
    b = S.Batcher(lay.engine, max_tokens=args.max_tokens)
    for s, q in reqs[:8]:
        lay.system_one(s, q, batcher=b)  # warm the worker
    b.stats.update(passes=0, questions=0, tokens=0)
    stop_at = [0.0]
    done = [0] * args.clients
    blat = [[] for _ in range(args.clients)]

    def client(c):
        j = c
        while time.perf_counter() < stop_at[0]:
            s, q = reqs[j % len(reqs)]
            t1 = time.perf_counter()
            lay.system_one(s, q, batcher=b)
            blat[c].append(time.perf_counter() - t1)
            done[c] += len(q)
            j += args.clients

    stop_at[0] = time.perf_counter() + args.seconds
    t = time.perf_counter()
    ths = [threading.Thread(target=client, args=(c,)) for c in range(args.clients)]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    wall = time.perf_counter() - t
    b.close()
    all_lat = [x for l_ in blat for x in l_]

    # many options: 64 questions of 120 options each (7,680 marker rows in gathered tiles) in one call
    rng = np.random.default_rng(120)
    many = []
    for i in range(64):
        crit = {"t%d" % (3000 + j): "queue t%d" % rng.integers(2000, 40000) for j in range(120)}
        state = " ".join("t%d" % v for v in rng.integers(2000, 40000, 300))
        many.append(lay.prepare(state, {"q": {"type": "choice", "instructions": "which queue?", "criteria": crit}})[2][0])
    ms, mm, mq = [x[0] for x in many], [x[1] for x in many], [x[2] for x in many]
    lay.engine.forward_batch(ms, mm, mq)
    t = time.perf_counter()
    for _ in range(reps):
        lay.engine.forward_batch(ms, mm, mq)
    many_rate = reps * len(many) / (time.perf_counter() - t)
    out = {
        "metric": "request-path decisions/sec (ModernBERT-large, C2 requests: state + 3 questions)",
        "workload": "C2 as requests: 64 states, L~U[32,512], 3 questions each (%d tokens)" % tokens,
        "devices": getattr(lay.engine, "num_devices", 1), "startup_s": round(startup, 2),
        "engine_only": {"decisions_per_s": round(eng_rate, 1), "call": "all %d questions in one forward_batch" % nq},
        "direct": {"decisions_per_s": round(direct_rate, 1), "p50_ms": round(pct(lat, 50), 3),
                   "p99_ms": round(pct(lat, 99), 3)},
        "batched": {"clients": args.clients, "seconds": round(wall, 2),
                    "decisions_per_s": round(sum(done) / wall, 1),
                    "p50_ms": round(pct(all_lat, 50), 2), "p99_ms": round(pct(all_lat, 99), 2),
                    "rounds": b.stats["passes"], "max_tokens": b.max_tokens,
                    "tokens_per_round": round(b.stats["tokens"] / max(1, b.stats["passes"]), 1),
                    "questions_per_round": round(b.stats["questions"] / max(1, b.stats["passes"]), 1)},
        "many_options": {"decisions_per_s": round(many_rate, 1), "questions": len(many), "options": 120,
                         "tokens_per_question": len(ms[0]), "call": "all questions in one forward_batch"},
        "host": {"prepare_ms_per_request": round(t_prep * 1e3, 3), "finish_ms_per_request": round(t_fin * 1e3, 3)},
        "graphs": os.environ.get("LAYA_GRAPHS", "1"),
    }
    print(json.dumps(out))
    lay.engine.close()


if __name__ == "__main__":
    main()
