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
from oracle import synth  # noqa: E402

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
