"""Request path end to end on the GPU: layamd_b200.server.Laya on the engine against the oracle's logits
pushed through the same finish(), directly and through the batching worker under concurrent requests."""
import json
import os
import threading

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from layamd_b200 import server as S  # noqa: E402
from oracle import model as om  # noqa: E402
from layamd_b200.synthetic import synth  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module", autouse=True)
def need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLD, "server_golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def tiny():
    ck = synth.checkpoint("tiny", 0)
    lay = S.Laya(ck, precision=1)  # fp32-parity engine; warm-up included
    yield ck, lay
    lay.engine.close()


def requests_of(golden):
    """The golden requests made for the tiny model's sequence budget (max_len 128, head_max_len 48)."""
    return [c for c in golden["cases"] if c["cfg"] == 0 and "error" not in c]


def oracle_answers(lay, ck, state, questions):
    o = om.Oracle(synth.load_weights(ck), synth.load_arch(ck))
    qids, qs, items = lay.prepare(state, questions)
    lo, ac, _ = o.forward_batch([{"ids": s, "markers": m, "qtype": t} for s, m, t in items])
    logits, off = [], 0
    for _, m, _ in items:
        logits.append(lo[off:off + len(m)].astype(np.float32))
        off += len(m)
    return lay.finish(qids, qs, items, logits, np.asarray(ac, np.float32), 0.0)


def close_answers(a, b, tol):
    assert a.keys() == b.keys()
    for qid in a:
        x, y = a[qid], b[qid]
        assert x["type"] == y["type"]
        assert abs(x["rl_agent"]["act_probability"] - y["rl_agent"]["act_probability"]) <= tol
        if x["type"] == "noul":
            assert abs(x["noul"] - y["noul"]) <= tol
            continue
        px, py = x["probabilities"], y["probabilities"]
        assert px.keys() == py.keys()
        assert max(abs(px[k] - py[k]) for k in px) <= tol, (qid, px, py)
        if x["type"] == "choice" and sorted(px.values())[-1] - sorted(px.values())[-2] > 2 * tol:
            assert x["choice"] == y["choice"]


def test_sequences_match_reference_layout(tiny, golden):
    """The checkpoint's own config and tokenizer give the token ids the reference's prepare gave."""
    _, lay = tiny
    for case in requests_of(golden):
        _, _, items = lay.prepare(case["state"], case["questions"])
        assert [[list(s), list(m), t] for s, m, t in items] == case["items"]


def test_answers_match_oracle(tiny, golden):
    ck, lay = tiny
    for case in requests_of(golden):
        got = lay.system_one(case["state"], case["questions"])
        want = oracle_answers(lay, ck, case["state"], case["questions"])
        assert got["usage"]["input_tokens"] == want["usage"]["input_tokens"]
        close_answers(got["answers"], want["answers"], 2e-4)


def test_batcher_rounds_match_direct_calls(tiny, golden):
    """Concurrent requests merged into rounds by the worker get the answers of their direct calls."""
    _, lay = tiny
    reqs = requests_of(golden) * 4
    direct = [lay.system_one(c["state"], c["questions"])["answers"] for c in reqs]
    b = S.Batcher(lay.engine, max_tokens=600)
    got = [None] * len(reqs)

    def client(t):
        for j in range(t, len(reqs), 6):
            got[j] = lay.system_one(reqs[j]["state"], reqs[j]["questions"], batcher=b)["answers"]

    ths = [threading.Thread(target=client, args=(t,)) for t in range(6)]
    for th in ths:
        th.start()
    for th in ths:
        th.join(120)
    b.close()
    assert b.stats["questions"] == sum(len(c["qids"]) for c in reqs)
    for a, d in zip(got, direct):
        close_answers(a, d, 2e-4)


# ---------------------------------------------------------------- many options (row f3)
@pytest.fixture(scope="module")
def large():
    ck = synth.checkpoint("large", 0)
    lay = S.Laya(ck, warmup=False)  # bf16 engine
    yield ck, lay
    lay.engine.close()


def many_option_requests():
    """Two 77-option and one 120-option choice questions (ticket routing style), 300-token states."""
    rng = np.random.default_rng(77)
    reqs = []
    for n in (77, 77, 120):
        crit = {"t%d" % (3000 + 7 * i + n): "queue t%d t%d" % tuple(rng.integers(2000, 40000, 2)) for i in range(n)}
        state = " ".join("t%d" % v for v in rng.integers(2000, 40000, 300))
        reqs.append((state, {"q": {"type": "choice", "instructions": "which queue should take this ticket?",
                                   "criteria": crit}}))
    return reqs


def test_many_options_match_oracle(large):
    """Questions with more options than one 64-row marker tile, all in one engine call (274 marker rows
    over several gathered tiles), on ModernBERT-large in bf16 through the request path: every
    probability within 0.01 of the fp32 oracle's and the same argmax wherever the oracle's top-2
    logit gap exceeds 2e-3 (the tolerance of the reference's many-option check,
    bench/eval/check_many_options.py)."""
    ck, lay = large
    o = om.Oracle(synth.load_weights(ck), synth.load_arch(ck))
    reqs = many_option_requests()
    prepared = [lay.prepare(s, q) for s, q in reqs]
    items = [it[0] for _, _, it in prepared]
    lg, ac = lay.engine.forward_batch([i[0] for i in items], [i[1] for i in items], [i[2] for i in items])
    lo_o, ac_o, _ = o.forward_batch([{"ids": s, "markers": m, "qtype": t} for s, m, t in items])
    off = 0
    for (qids, qs, it), got in zip(prepared, lg):
        k = len(it[0][1])
        want = np.asarray(lo_o[off:off + k], np.float64)
        off += k
        assert len(got) == k == len(qs[0]["crit"])
        pg, pw = S._softmax(np.asarray(got, np.float64)), S._softmax(want)
        assert np.abs(pg - pw).max() < 0.01
        top = np.sort(want)[::-1]
        if top[0] - top[1] > 2e-3:
            assert int(np.argmax(got)) == int(np.argmax(want))
    assert np.abs(np.asarray(ac, np.float64) - np.asarray(ac_o, np.float64)).max() < 0.05 * np.abs(ac_o).max()
    # the same questions as requests give the same probabilities as the single call
    for (s, q), (qids, qs, it), got in zip(reqs, prepared, lg):
        ans = lay.system_one(s, q)["answers"]["q"]["probabilities"]
        p = S._softmax(np.asarray(got, np.float64) / lay.temperature[0])
        assert max(abs(ans[kk] - float(v)) for kk, v in zip(qs[0]["crit"], p)) <= 2e-3
