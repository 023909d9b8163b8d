"""Request path (layamd_b200.server) on CPU: parity with the reference's own prepare / finish over the
committed golden requests (tests/golden/make_server_golden.py), and the batching worker's contract
with a fake engine (no GPU, no library)."""
import json
import os
import shutil
import threading
import time

import numpy as np
import pytest

from layamd_b200 import server as S

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


class FakeEngine:
    """forward_batch with a deterministic function of each sequence: logit j = (sum of ids + 7 j) mod 97
    / 10, act = [len / 100, qtype]. Records every call's sizes; optionally sleeps or fails."""

    def __init__(self, max_markers=255, delay=0.0, fail_on=None, num_devices=1):
        self.max_markers, self.delay, self.fail_on, self.num_devices = max_markers, delay, fail_on, num_devices
        self.calls = []
        self.lock = threading.Lock()

    @staticmethod
    def expect(seq, markers, qtype):
        s = int(np.sum(seq))
        lg = np.array([((s + 7 * j) % 97) / 10.0 for j in range(len(markers))], np.float32)
        return lg, np.array([len(seq) / 100.0, float(qtype)], np.float32)

    def forward_batch(self, seqs, markers, qtypes):
        with self.lock:
            self.calls.append((len(seqs), sum(len(s) for s in seqs)))
        if self.delay:
            time.sleep(self.delay)
        if self.fail_on is not None and any(self.fail_on in s for s in seqs):
            raise ValueError("engine rejected batch (sequence too long or too many options)")
        out = [self.expect(s, m, t) for s, m, t in zip(seqs, markers, qtypes)]
        return [o[0] for o in out], np.stack([o[1] for o in out]) if out else np.zeros((0, 2), np.float32)


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLD, "server_golden.json")) as f:
        return json.load(f)


def make_laya(tmp_path, cfg, engine):
    d = tmp_path / ("ck%d" % abs(hash(json.dumps(cfg, sort_keys=True))))
    if not d.exists():
        d.mkdir()
        shutil.copytree(os.path.join(GOLD, "server_tok"), str(d / "tokenizer"))
        (d / "rl_agent_config.json").write_text(json.dumps(cfg))
    return S.Laya(str(d), engine=engine, warmup=False)


def test_golden_prepare_and_finish(tmp_path, golden):
    """Every golden request: the same qids, token ids, markers and qtypes as the reference's prepare (or
    the same error), and the same answers as the reference's finish for the stored logits."""
    for i, case in enumerate(golden["cases"]):
        lay = make_laya(tmp_path, golden["cfgs"][case["cfg"]], FakeEngine(max_markers=case["max_markers"]))
        if "error" in case:
            with pytest.raises(ValueError) as e:
                lay.prepare(case["state"], case["questions"])
            assert str(e.value) == case["error"], i
            continue
        qids, qs, items = lay.prepare(case["state"], case["questions"])
        assert qids == case["qids"], i
        assert [[list(s), list(m), t] for s, m, t in items] == case["items"], i
        logits = [np.array(lg, np.float32) for lg in case["logits"]]
        act = np.array(case["act"], np.float32).reshape(len(items), -1) if items else np.zeros((0, 3), np.float32)
        out = lay.finish(qids, qs, items, logits, act, time.perf_counter())
        assert out["usage"].pop("latency_ms") >= 0
        assert out == case["result"], i


def test_batched_header_tokenisation_matches_single(tmp_path, golden):
    lay = make_laya(tmp_path, golden["cfgs"][0], FakeEngine())
    texts = ["choice question: which way?", "", "noul question: the door is open {\"a\": [1, 2]}", "zebra " * 50]
    assert lay.tok.ids_batch(texts) == [lay.tok.ids(t) for t in texts]


def test_system_one_direct_and_empty(tmp_path, golden):
    eng = FakeEngine()
    lay = make_laya(tmp_path, golden["cfgs"][1], eng)
    case = golden["cases"][4]
    out = lay.system_one(case["state"], case["questions"])
    assert list(out["answers"]) == case["qids"]
    assert out["usage"]["input_tokens"] == sum(len(it[0]) for it in case["items"])
    assert len(eng.calls) == 1
    empty = lay.system_one("nothing", {})
    assert empty["answers"] == {} and empty["usage"]["input_tokens"] == 0
    assert len(eng.calls) == 1  # no engine call for a request without questions


def _items(rng, n, lo=5, hi=60):
    out = []
    for _ in range(n):
        L = int(rng.integers(lo, hi))
        k = int(rng.integers(2, 5))
        out.append((list(rng.integers(0, 900, L)), sorted(rng.choice(np.arange(1, L), k, replace=False).tolist()),
                    int(rng.integers(0, 3))))
    return out


def test_batcher_concurrent_requests_get_their_own_results():
    eng = FakeEngine(delay=0.005)
    b = S.Batcher(eng, max_tokens=400)
    rng = np.random.default_rng(3)
    reqs = [_items(rng, int(rng.integers(1, 4))) for _ in range(48)]
    results = [None] * len(reqs)

    def client(idx):
        for j in range(idx, len(reqs), 8):
            results[j] = b.run(reqs[j])

    threads = [threading.Thread(target=client, args=(t,)) for t in range(8)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(30)
    b.close()
    for req, (lg, ac) in zip(reqs, results):
        for it, l_, a_ in zip(req, lg, ac):
            el, ea = FakeEngine.expect(*it)
            assert np.array_equal(l_, el) and np.array_equal(a_, ea)
    assert b.stats["questions"] == sum(len(r) for r in reqs)
    assert b.stats["passes"] == len(eng.calls) < len(reqs)  # rounds did merge requests
    # a round exceeds the budget only when its first request alone does
    biggest = max(sum(len(it[0]) for it in r) for r in reqs)
    assert all(tok <= max(400, biggest) for _, tok in eng.calls)


def test_batcher_budget_and_carry():
    """With the worker busy, queued requests form rounds of at most max_tokens tokens in arrival order;
    the one that does not fit leads the next round."""
    eng = FakeEngine(delay=0.05)
    b = S.Batcher(eng, max_tokens=100)
    rng = np.random.default_rng(4)
    first = _items(rng, 1, 90, 91)
    t0 = threading.Thread(target=b.run, args=(first,))
    t0.start()
    time.sleep(0.01)  # the worker is now inside the first round's engine call
    reqs = [[(list(range(40)), [1, 2], 0)] for _ in range(5)]  # 40 tokens each: two per round
    outs = [None] * 5

    def go(i):
        outs[i] = b.run(reqs[i])

    ths = []
    for i in range(5):
        th = threading.Thread(target=go, args=(i,))
        th.start()
        ths.append(th)
        time.sleep(0.002)  # keep arrival order
    for th in ths + [t0]:
        th.join(30)
    b.close()
    assert [c for c in eng.calls] == [(1, 90), (2, 80), (2, 80), (1, 40)]
    assert all(o is not None for o in outs)


def test_batcher_default_budget_scales_with_gpus():
    b = S.Batcher(FakeEngine(num_devices=4))
    assert b.max_tokens == 4 * S.DEFAULT_PASS_TOKENS
    b.close()


def test_batcher_engine_error_fails_only_its_round():
    eng = FakeEngine(delay=0.02, fail_on=999)
    b = S.Batcher(eng, max_tokens=10_000)
    bad = [([1, 999, 3, 4], [1, 2], 0)]
    good = [([1, 2, 3, 4], [1, 2], 0)]
    errs = []

    def run(items):
        try:
            b.run(items)
        except ValueError as e:
            errs.append(str(e))

    t1 = threading.Thread(target=run, args=(bad,))
    t1.start()
    t1.join(10)
    assert errs == ["engine rejected batch (sequence too long or too many options)"]
    lg, ac = b.run(good)  # the worker survives and serves the next round
    assert np.array_equal(lg[0], FakeEngine.expect(*good[0])[0])
    b.close()
