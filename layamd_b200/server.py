"""Decision request path above the engine: sequence construction, per-request prepare / finish and
continuous batching across concurrent requests, on ``liblaya_b200.so``.

This is the caller side of ``laya_forward_batch`` in the reference's server
(mauimauer/layamd server/laya_server.py:53-242): a request is a state plus named questions; each
question becomes one token sequence ``[CLS] <type> question: <ins> [SEP] [MASK] opt0 [MASK] opt1 ...
[SEP] state [SEP]`` with a marker at every ``[MASK]``; the engine returns one raw logit per marker and
the act logits per question; the answers are the temperature-scaled softmax over the options. The
sequence layout, truncation rules, temperature buckets and answer format are the reference's (the
checkpoints were trained on that layout and its clients parse that format); the HTTP layer is not
part of this module.

B200 choices: the batching worker hands the engine rounds of up to 65536 tokens per GPU of the
handle instead of 4096 tokens (a B200 pass reaches its full rate at about 16k tokens; 65536 keeps a
round's latency near one C2-size pass), so concurrent requests share passes on every GPU; a request's
question headers are tokenised in one batched call; and the worker can be stopped
(``Batcher.close``).
"""
import collections
import functools
import itertools
import json
import math
import os
import threading
import time
from concurrent.futures import Future
from dataclasses import dataclass, field
from typing import Deque, Dict, List, Optional, Sequence, Tuple

import numpy as np

QTYPES = {"choice": 0, "score": 1, "noul": 2}
QTYPE_NAMES = {v: k for k, v in QTYPES.items()}
OPTION_TOKENS = 48  # tokens kept per rendered option after its [MASK] (laya_server.py:79)
DEFAULT_PASS_TOKENS = 65536  # tokens per GPU per batching round


# ------------------------------------------------------------------ sequence construction
def serialize_state(state) -> str:
    """A state is text, or any JSON value serialised without ASCII escaping (laya_server.py:54-55)."""
    if isinstance(state, str):
        return state
    return json.dumps(state, ensure_ascii=False)


def render_options(q: Dict) -> List[str]:
    """The option strings of an internal question (laya_server.py:57-65): choice options are their
    keys, or "key: description"; score levels are "level i: text"; a yes/no question has a false and
    a true option with default wording."""
    kind, crit = q["t"], q.get("crit")
    if kind == "choice":
        return [name if not desc else "%s: %s" % (name, desc) for name, desc in crit.items()]
    if kind == "score":
        return ["level %d: %s" % (i, text) for i, text in enumerate(crit)]
    crit = crit or {}
    false_text = crit.get("false") or "no, the statement does not hold"
    true_text = crit.get("true") or "yes, the statement holds"
    return ["false: " + false_text, "true: " + true_text]


class Tok:
    """Tokenizer of a checkpoint (``tokenizer/tokenizer.json`` + ``tokenizer_config.json``): the
    special-token ids and the option encoding of laya_server.py:67-80."""

    def __init__(self, path: str, cfg_path: str):
        from tokenizers import Tokenizer  # the Rust tokenizers library, as the reference server uses

        self.t = Tokenizer.from_file(path)
        cfg = {}
        if os.path.exists(cfg_path):
            with open(cfg_path) as f:
                cfg = json.load(f)
        self.mask_token = cfg.get("mask_token", "[MASK]")
        self.mask_token_id = self.t.token_to_id(self.mask_token)
        self.cls_token_id = self.t.token_to_id(cfg.get("cls_token", "[CLS]"))
        self.sep_token_id = self.t.token_to_id(cfg.get("sep_token", "[SEP]"))
        self.pad_token_id = self.t.token_to_id(cfg.get("pad_token", "[PAD]"))
        self.opt_ids = functools.lru_cache(maxsize=512)(self._opt_ids)

    def ids(self, text: str) -> List[int]:
        return self.t.encode(text, add_special_tokens=False).ids

    def ids_batch(self, texts: Sequence[str]) -> List[List[int]]:
        """Same ids as ``ids`` per text, encoded by the library's thread pool in one call."""
        return [e.ids for e in self.t.encode_batch(list(texts), add_special_tokens=False)]

    def _opt_ids(self, option: str) -> Tuple[int, ...]:
        body = self.ids(" " + option.replace(self.mask_token, " "))[:OPTION_TOKENS]
        return (self.mask_token_id,) + tuple(body)


def header_text(tok: Tok, q: Dict) -> str:
    return "%s question: %s" % (q["t"], str(q["ins"]).replace(tok.mask_token, " "))


def build_sequence(tok: Tok, state, q: Dict, max_len: int, head_max_len: int,
                   state_ids: Optional[List[int]] = None, opts: Optional[List[str]] = None,
                   head_ids: Optional[List[int]] = None):
    """Token ids and marker positions of one question (laya_server.py:82-107).

    The header and options share ``head_max_len`` tokens: if fewer than 16 would remain for the
    header, every option is cut to max(4, (head_max_len - 16) / #options) tokens; the header keeps at
    least 8. The state fills what is left of ``max_len`` before the closing [SEP]; markers past
    ``max_len`` are dropped (the caller treats that as an error)."""
    if opts is None:
        opts = render_options(q)
    if head_ids is None:
        head_ids = tok.ids(header_text(tok, q))
    option_ids = [tok.opt_ids(o) for o in opts]
    budget = head_max_len - sum(len(o) for o in option_ids)
    if budget < 16:
        keep = max(4, (head_max_len - 16) // max(1, len(option_ids)))
        option_ids = [o[:keep] for o in option_ids]
        budget = head_max_len - sum(len(o) for o in option_ids)
    seq = [tok.cls_token_id]
    seq.extend(head_ids[:max(8, budget)])
    seq.append(tok.sep_token_id)
    markers = []
    for o in option_ids:
        markers.append(len(seq))
        seq.extend(o)
    seq.append(tok.sep_token_id)
    room = max(0, max_len - len(seq) - 1)
    if state_ids is None:
        state_ids = tok.ids(serialize_state(state).replace(tok.mask_token, " "))
    seq.extend(state_ids[:room])
    seq.append(tok.sep_token_id)
    return seq[:max_len], [m for m in markers if m < max_len]


def temp_bucket(qtype: int, k: int) -> str:
    """Key of ``temperature_by_options`` for a question type and option count (laya_server.py:109-111)."""
    if k <= 2:
        size = "2"
    elif k <= 5:
        size = "3-5"
    elif k <= 10:
        size = "6-10"
    else:
        size = "11+"
    return "%s:%s" % (QTYPE_NAMES[int(qtype)], size)


def confidence_from_probs(p, k: int) -> float:
    """1 - H(p) / log k over the first k probabilities; 1 for fewer than two options."""
    if k < 2:
        return 1.0
    p = p[:k]
    entropy = -(p * np.log(np.clip(p, 1e-12, 1))).sum()
    return float(1 - entropy / math.log(k))


def _softmax(z):
    e = np.exp(z - z.max())
    return e / e.sum()


# ------------------------------------------------------------------ requests
class Laya:
    """Decisions for (state, questions) requests: the reference server's ``Laya`` class
    (laya_server.py:124-188) on this engine.

    ``engine``: an ``layamd_b200.Engine`` (or any object with ``forward_batch`` and ``max_markers``);
    created from ``model_dir`` when omitted. ``warmup`` captures the single-question graphs the way
    the reference server does at start-up."""

    def __init__(self, model_dir: str, engine=None, precision: int = 0, devices: str = "", warmup: bool = True):
        with open(os.path.join(model_dir, "rl_agent_config.json")) as f:
            self.cfg = json.load(f)
        self.tok = Tok(os.path.join(model_dir, "tokenizer", "tokenizer.json"),
                       os.path.join(model_dir, "tokenizer", "tokenizer_config.json"))
        if engine is None:
            from . import Engine

            engine = Engine(model_dir, precision=precision, devices=devices)
        self.engine = engine
        self.temperature = self.cfg.get("temperature", [1.0, 1.0, 1.0])
        self.temp_by_options = self.cfg.get("temperature_by_options", {})
        self.model_name = self.cfg.get("model_name", "laya")
        if warmup:
            self.warmup()

    def warmup(self):
        """Tunes the engine and runs one single-question call per 64-token length step, so the first
        requests do not pay for graph capture."""
        if hasattr(self.engine, "tune_all"):
            self.engine.tune_all()
        for n in range(64, int(self.cfg["max_len"]) + 1, 64):
            self.engine.forward_batch([[self.tok.cls_token_id] * n], [[1, 2]], [0])

    @staticmethod
    def _to_internal(qdef: Dict) -> Dict:
        kind, crit = qdef["type"], qdef.get("criteria")
        if kind == "choice" and isinstance(crit, list):
            crit = {c: None for c in crit}
        ins = qdef["instructions"]
        return {"t": kind, "crit": crit, "ins": ins if isinstance(ins, str) else json.dumps(ins)}

    def prepare(self, state, questions: Dict):
        """Tokenises the state once and builds every question's sequence. Raises ValueError for a
        question whose options do not fit ``head_max_len`` or that has more options than the engine
        accepts (laya_server.py:143-161)."""
        qids, qs, items = [], [], []
        if not questions:
            return qids, qs, items
        tok = self.tok
        state_ids = tok.ids(serialize_state(state).replace(tok.mask_token, " "))
        max_len, head_max_len = self.cfg["max_len"], self.cfg["head_max_len"]
        internal = [(qid, self._to_internal(qdef)) for qid, qdef in questions.items()]
        headers = tok.ids_batch([header_text(tok, q) for _, q in internal])
        for (qid, q), head_ids in zip(internal, headers):
            opts = render_options(q)
            seq, markers = build_sequence(tok, state, q, max_len, head_max_len, state_ids=state_ids, opts=opts,
                                          head_ids=head_ids)
            if len(markers) != len(opts):
                raise ValueError("question %r: options do not fit in head_max_len=%d tokens" % (qid, head_max_len))
            if len(markers) > self.engine.max_markers:
                raise ValueError("question %r: more than %d options" % (qid, self.engine.max_markers))
            qids.append(qid)
            qs.append(q)
            items.append((seq, markers, QTYPES[q["t"]]))
        return qids, qs, items

    def finish(self, qids, qs, items, logits, act, t0) -> Dict:
        """Answers from the raw logits (laya_server.py:163-188): probabilities = softmax(logits / T)
        with T from ``temperature_by_options`` (type and option-count bucket) or the per-type
        temperature; the act probability is the first entry of softmax(act logits)."""
        answers = {}
        for qid, q, (_, _, qt), lg, ac in zip(qids, qs, items, logits, act):
            k = len(lg)
            p = _softmax(lg / self.temp_by_options.get(temp_bucket(qt, k), self.temperature[qt]))
            ext = {"act_probability": float(_softmax(ac)[0])}
            if q["t"] == "choice":
                keys = list(q["crit"].keys())
                answers[qid] = {"type": "choice", "choice": keys[int(p.argmax())],
                                "probabilities": {name: round(float(v), 4) for name, v in zip(keys, p)},
                                "confidence": round(confidence_from_probs(p, k), 4), "rl_agent": ext}
            elif q["t"] == "score":
                answers[qid] = {"type": "score", "score": round(float((np.arange(k) * p).sum()), 4),
                                "legend": {str(i): c for i, c in enumerate(q["crit"])},
                                "probabilities": {str(i): round(float(v), 4) for i, v in enumerate(p)},
                                "confidence": round(confidence_from_probs(p, k), 4), "rl_agent": ext}
            else:
                answers[qid] = {"type": "noul", "noul": round(float(p[1]), 4), "rl_agent": ext}
        return {"model": self.model_name, "answers": answers,
                "usage": {"input_tokens": sum(len(it[0]) for it in items), "output_tokens": 0,
                          "latency_ms": round((time.perf_counter() - t0) * 1000, 2)}}

    def system_one(self, state, questions: Dict, batcher: Optional["Batcher"] = None) -> Dict:
        """One request: prepare, one engine call (through ``batcher`` when given), finish."""
        t0 = time.perf_counter()
        qids, qs, items = self.prepare(state, questions)
        if not items:
            return self.finish(qids, qs, items, [], [], t0)
        if batcher is not None:
            logits, act = batcher.run(items)
        else:
            logits, act = self.engine.forward_batch([i[0] for i in items], [i[1] for i in items],
                                                    [i[2] for i in items])
        return self.finish(qids, qs, items, logits, act, t0)


@dataclass
class _Ticket:
    """One request's questions waiting for a round, and the future its caller blocks on."""
    seqs: List[List[int]]
    markers: List[List[int]]
    qtypes: List[int]
    tokens: int
    result: Future = field(default_factory=Future)


class Batcher:
    """Continuous batching of concurrent requests into engine rounds.

    Requests are queued as tickets; a single serving thread takes the oldest pending tickets, as many
    as fit ``max_tokens`` tokens (never splitting a request; one larger than the budget runs alone),
    and makes ONE ``forward_batch`` call for them: the engine packs the round back to back and, on a
    multi-GPU handle, shards it over its replicas. Tickets that arrive while a round runs, or that did
    not fit it, stay queued in arrival order for the next round. Each caller waits on its ticket's
    future; if the engine call raises, every ticket of that round receives the exception and the
    thread goes on serving. The observable rules (a token budget per round, arrival order, one call
    per round, an error fails its whole round) are the reference server's worker
    (server/laya_server.py:191-242); the structure here is its own.

    ``max_tokens`` defaults to DEFAULT_PASS_TOKENS per GPU of the engine (``num_devices``), so one
    round fills every GPU's pass."""

    def __init__(self, engine, max_tokens: Optional[int] = None):
        if max_tokens is None:
            max_tokens = DEFAULT_PASS_TOKENS * max(1, int(getattr(engine, "num_devices", 1) or 1))
        self.engine, self.max_tokens = engine, int(max_tokens)
        self.stats = {"passes": 0, "questions": 0, "tokens": 0}
        self._pending: Deque[_Ticket] = collections.deque()
        self._cv = threading.Condition()
        self._closing = False
        self._server = threading.Thread(target=self._serve, daemon=True, name="laya-batcher")
        self._server.start()

    def submit(self, items) -> Future:
        """Queues one request's questions (``(token ids, markers, qtype)`` each); the future resolves to
        (per-question logits, act rows) once its round has run."""
        t = _Ticket([it[0] for it in items], [it[1] for it in items], [it[2] for it in items],
                    sum(len(it[0]) for it in items))
        with self._cv:
            if self._closing:
                raise RuntimeError("batcher is closed")
            self._pending.append(t)
            self._cv.notify()
        return t.result

    def run(self, items):
        """Blocks until the round holding ``items`` has run; returns (per-question logits, act rows)."""
        return self.submit(items).result()

    def close(self, timeout: float = 10.0):
        """Refuses new requests, serves the ones already queued, then stops the serving thread."""
        with self._cv:
            self._closing = True
            self._cv.notify()
        self._server.join(timeout)

    def _take_round(self) -> Optional[List[_Ticket]]:
        with self._cv:
            self._cv.wait_for(lambda: self._pending or self._closing)
            if not self._pending:
                return None  # closed and drained
            taken = [self._pending.popleft()]
            budget = self.max_tokens - taken[0].tokens
            while self._pending and self._pending[0].tokens <= budget:
                budget -= self._pending[0].tokens
                taken.append(self._pending.popleft())
            return taken

    def _serve(self):
        while True:
            tickets = self._take_round()
            if tickets is None:
                return
            seqs = list(itertools.chain.from_iterable(t.seqs for t in tickets))
            marks = list(itertools.chain.from_iterable(t.markers for t in tickets))
            qts = list(itertools.chain.from_iterable(t.qtypes for t in tickets))
            try:
                logits, act = self.engine.forward_batch(seqs, marks, qts)
            except Exception as e:  # the whole round fails with the engine's error
                for t in tickets:
                    t.result.set_exception(e)
                continue
            self.stats["passes"] += 1
            self.stats["questions"] += len(seqs)
            self.stats["tokens"] += sum(t.tokens for t in tickets)
            lo = 0
            for t in tickets:
                hi = lo + len(t.seqs)
                t.result.set_result((list(logits[lo:hi]), list(act[lo:hi])))
                lo = hi
