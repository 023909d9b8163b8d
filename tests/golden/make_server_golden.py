"""Generates tests/golden/server_golden.json (and the tokenizer in tests/golden/server_tok/) from the
reference's own request code (test infrastructure).

Run in the build container, where the reference checkout is available (LAYA_REFERENCE):

    python tests/golden/make_server_golden.py

It imports the reference's server/laya_server.py in place and drives ``Laya.prepare`` and
``Laya.finish`` (server/laya_server.py:143-188) on an instance built without its engine (only
``max_markers`` of the engine is read by those two methods), with the synthetic word-level tokenizer
of the tiny checkpoint (layamd_b200/synthetic/synth.py ``write_tokenizer``), over requests chosen to reach every
branch of the sequence construction (server/laya_server.py:82-107): list / dict / described choice
criteria, score levels, yes/no with and without custom wording, JSON states and instructions,
[MASK] inside texts, states longer than max_len, many options (per-option truncation), options that
no longer fit (error), more options than the engine accepts (error) and an empty request. For every
prepared request it stores seeded logits and act logits and the reference's answers for them
(latency removed). The tests compare layamd_b200.server against this file on CPU; the GPU boxes only
read the committed JSON.
"""
import json
import os
import sys
import types

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from layamd_b200.synthetic import synth  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
from oracle.ref_tools import reference_root  # noqa: E402

REF = reference_root()
TOK_DIR = os.path.join(HERE, "server_tok")

CFGS = [
    {"max_len": 128, "head_max_len": 48, "temperature": [0.7, 1.3, 2.0],
     "temperature_by_options": {"choice:3-5": 0.5, "score:3-5": 1.7, "noul:2": 0.9}, "model_name": "laya-tiny"},
    {"max_len": 512, "head_max_len": 192, "temperature": [1.0, 1.0, 1.0], "model_name": "laya"},
]

LONG_STATE = " ".join("step %d the agent is in room %d and the door is open" % (i, i % 7) for i in range(80))
MANY = ["option %d with quite a lot of words describing what the agent should do next" % i for i in range(12)]


def requests():
    r = []
    r.append((0, 255, "the door is open", {"q1": {"type": "choice", "instructions": "which action is best?",
                                                  "criteria": ["go", "wait", "stop"]}}))
    r.append((0, 255, {"room": "kitchen", "items": ["key", "box"], "note": "café – ok"},
              {"pick": {"type": "choice", "instructions": "what should the agent pick up?",
                        "criteria": {"key": "the red key on the table", "box": None, "chair": ""}},
               "rate": {"type": "score", "instructions": {"task": "rate the answer", "scale": [0, 1, 2]},
                        "criteria": ["bad answer", "good answer", "correct and helpful answer"]},
               "safe": {"type": "noul", "instructions": "is the room safe?"}}))
    r.append((0, 255, LONG_STATE, {"open": {"type": "noul", "instructions": "the door is [MASK] open",
                                             "criteria": {"true": "yes it is open", "false": None}},
                                    "move": {"type": "choice", "instructions": "move [MASK] where?",
                                             "criteria": ["left [MASK]", "right", "up", "down", "wait"]}}))
    r.append((0, 255, "short", {"many": {"type": "choice", "instructions": "pick one " * 30,
                                           "criteria": MANY[:6]}}))
    r.append((1, 255, LONG_STATE, {"many": {"type": "choice", "instructions": "which option is best for the user",
                                             "criteria": MANY},
                                    "lvl": {"type": "score", "instructions": "rate the quality",
                                            "criteria": ["low", "high"]}}))
    r.append((0, 255, "x", {"toomany": {"type": "choice", "instructions": "pick",
                                         "criteria": ["choose option %d now" % i for i in range(40)]}}))
    r.append((1, 8, "x", {"limit": {"type": "choice", "instructions": "pick",
                                     "criteria": ["o%d" % i for i in range(10)]}}))
    r.append((1, 255, "nothing to ask", {}))
    r.append((1, 255, "unknown words zebra quantum fjord", {"u": {"type": "noul", "instructions": "zebra?",
                                                                  "criteria": {"true": "", "false": "nope"}}}))
    return r


def main():
    synth.write_tokenizer(TOK_DIR, synth.ARCHS["tiny"])
    sys.path.insert(0, os.path.join(REF, "server"))
    import laya_server as R  # the reference's request code

    tok = R.Tok(os.path.join(TOK_DIR, "tokenizer.json"), os.path.join(TOK_DIR, "tokenizer_config.json"))
    rng = np.random.default_rng(7)
    cases = []
    for ci, max_markers, state, questions in requests():
        lay = R.Laya.__new__(R.Laya)
        cfg = CFGS[ci]
        lay.cfg, lay.tok = cfg, tok
        lay.engine = types.SimpleNamespace(max_markers=max_markers)
        lay.temperature = cfg.get("temperature", [1.0, 1.0, 1.0])
        lay.temp_by_options = cfg.get("temperature_by_options", {})
        lay.model_name = cfg.get("model_name", "laya")
        case = {"cfg": ci, "max_markers": max_markers, "state": state, "questions": questions}
        try:
            qids, qs, items = lay.prepare(state, questions)
        except ValueError as e:
            case["error"] = str(e)
            cases.append(case)
            continue
        case["qids"] = qids
        case["items"] = [[list(map(int, s)), list(map(int, m)), int(t)] for s, m, t in items]
        logits = [(3 * rng.standard_normal(len(m))).astype(np.float32) for _, m, _ in items]
        act = (2 * rng.standard_normal((len(items), 3))).astype(np.float32)
        out = lay.finish(qids, qs, items, logits, act, 0.0)
        del out["usage"]["latency_ms"]
        case["logits"] = [lg.tolist() for lg in logits]
        case["act"] = act.tolist()
        case["result"] = out
        cases.append(case)
    with open(os.path.join(HERE, "server_golden.json"), "w") as f:
        json.dump({"cfgs": CFGS, "cases": cases}, f, indent=0, ensure_ascii=False)
    print("wrote %d cases" % len(cases))


if __name__ == "__main__":
    main()
