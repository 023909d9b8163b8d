"""Shared helpers of the engine tests: handles, batches through the C ABI, per-layer dumps and the
comparison metrics of the parity contract.

Metrics: hidden states use max|a-b| / max|b| over the whole layer tensor (the reference probes'
definition, bench/probes/wgemm_bench.cpp:25-27); probabilities are the per-question softmax of the
raw logits at temperature 1 (src/test_parity.cpp:60-65); act logits use |a-b| / max(1, |b|)
(src/test_parity.cpp:282-283).
"""
import ctypes
import os
import tempfile

import numpy as np

from layamd_b200 import PRECISION_BF16, PRECISION_FP32_PARITY, load_lib  # noqa: F401
from layamd_b200.synthetic import workloads

IP = ctypes.POINTER(ctypes.c_int)
FP = ctypes.POINTER(ctypes.c_float)


class Handle:
    def __init__(self, ckpt, precision=0, devices="", env=None):
        old = {}
        for k, v in (env or {}).items():
            old[k] = os.environ.get(k)
            os.environ[k] = str(v)
        try:
            self.L = load_lib()
            self.h = self.L.laya_create_ex(ckpt.encode(), precision, devices.encode() if devices else None)
        finally:
            for k, v in old.items():
                if v is None:
                    os.environ.pop(k, None)
                else:
                    os.environ[k] = v
        assert self.h, "laya_create_ex failed for %s" % ckpt
        self.n_act = self.L.laya_n_act(self.h)

    def close(self):
        if self.h:
            self.L.laya_destroy(self.h)
            self.h = None

    def forward(self, qs, dump_dir=None):
        """Returns (rc, logits, act) for a list of questions, optionally dumping per-layer tensors."""
        lens, ids, nmark, markers, qtypes = workloads.flatten(qs)
        lo = np.full(max(1, int(nmark.sum())), np.nan, np.float32)
        ac = np.full((max(1, len(qs)), self.n_act), np.nan, np.float32)
        self.L.laya_set_dump_dir(self.h, dump_dir.encode() if dump_dir else None)
        p = lambda a: a.ctypes.data_as(IP)  # noqa: E731
        rc = self.L.laya_forward_batch(self.h, len(qs), p(lens), p(ids if ids.size else np.zeros(1, np.int32)),
                                       p(nmark), p(markers if markers.size else np.zeros(1, np.int32)), p(qtypes),
                                       lo.ctypes.data_as(FP), ac.ctypes.data_as(FP))
        self.L.laya_set_dump_dir(self.h, None)
        return rc, lo[:int(nmark.sum())], ac[:len(qs)]

    def forward_dump(self, qs):
        d = tempfile.mkdtemp(prefix="laya_dump_")
        rc, lo, ac = self.forward(qs, d)
        assert rc == 0, rc
        return lo, ac, d


def read_dump(d, name, D):
    a = np.fromfile(os.path.join(d, name + ".bin"), dtype=np.float32)
    return a.reshape(-1, D)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def per_question(flat, qs):
    out, o = [], 0
    for q in qs:
        k = len(q["markers"])
        out.append(flat[o:o + k])
        o += k
    return out


def softmax(z):
    z = np.asarray(z, np.float64)
    e = np.exp(z - z.max())
    return e / e.sum()


def prob_delta(lo_a, lo_b, qs):
    return max(float(np.abs(softmax(a) - softmax(b)).max()) for a, b in zip(per_question(lo_a, qs), per_question(lo_b, qs)))


ARGMAX_MARGIN = 2e-3


def argmax_agree(lo_a, lo_b, qs, margin=ARGMAX_MARGIN):
    """bf16 argmax rule: the engine's argmax equals the reference's for every question whose reference
    top-1 minus top-2 logit gap exceeds `margin` (2e-3, several times the bf16 logit error); closer
    near-ties -- common with random-init weights, whose option logits often differ by 1e-4 -- are not
    decidable at bf16 precision and only enter the probability-delta check."""
    for a, b in zip(per_question(lo_a, qs), per_question(lo_b, qs)):
        if len(b) < 2:
            continue
        top = np.sort(np.asarray(b, np.float64))[::-1]
        if top[0] - top[1] > margin and int(np.argmax(a)) != int(np.argmax(b)):
            return False
    return True


def act_rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float((np.abs(a - b) / np.maximum(1.0, np.abs(b))).max())


def gathered_rows(caps_key, qs, caps):
    """Rows of the last head layer as the engine lays them out: every question's markers, then CLS."""
    marks = [c[caps_key][np.asarray(q["markers"])] for c, q in zip(caps, qs)]
    cls = [c[caps_key][0:1] for c in caps]
    return np.concatenate(marks + cls)
