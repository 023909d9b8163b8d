"""Checks this engine against a golden set written by the reference's ref/gen_golden.py.

    python -m layamd_b200.golden_parity MODEL_DIR GOLDEN_DIR [--precision bf16|fp32parity] [--devices 0]

The counterpart of the reference's src/test_parity.cpp (same inputs, same per-row report and
verdict), extended by the per-layer comparison the golden files make possible. GOLDEN_DIR holds
manifest.json and one directory per case with the padded batch the reference ran
(ref/gen_golden.py:72-105): int32 input_ids / attention_mask [n, L], marker_pos / marker_mask
[n, K], qtype [n]; fp32 logits [n, K], act_logits [n, n_act] and the hooked hidden states emb,
enc<i>, final_norm, head0, head1 [n, L, D].

Each case runs as ONE laya_forward_batch call over its valid tokens, twice: first with the engine's
per-layer dumps on (eager launches), then again as a graph replay, as test_parity.cpp does. Per
row: max |dlogit|, max |dprob| (softmax over the question's options) and the act logits' relative
error, passing at |dprob| < 0.01 and rel |dact| < 0.05 (src/test_parity.cpp:61-69). In fp32parity
mode the stricter bounds apply as well: |dprob| <= 1e-4, and max |a - b| / max |b| <= 1e-3 for every
hooked layer over the sequences' valid rows (the last head layer at the rows the engine computes:
every marker, then each question's first row). The API answers stored in the manifest are compared
with the probabilities the engine's logits give at the model's temperatures (to their 4 decimals).
"""
import argparse
import json
import os
import shutil
import struct
import sys
import tempfile
from typing import Dict, List, Optional

import numpy as np

QTYPE_NAMES = ("choice", "score", "noul")


def _softmax(z):
    z = np.asarray(z, np.float64)
    e = np.exp(z - z.max())
    return e / e.sum()


def read_tensor(path: str, name: str) -> np.ndarray:
    """One tensor of a safetensors file as fp32 (F32, BF16 or F16)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        meta = header[name]
        a, b = meta["data_offsets"]
        f.seek(8 + n + a)
        raw = f.read(b - a)
    dt = meta["dtype"]
    if dt == "F32":
        arr = np.frombuffer(raw, np.float32)
    elif dt == "F16":
        arr = np.frombuffer(raw, np.float16).astype(np.float32)
    elif dt == "BF16":
        arr = (np.frombuffer(raw, np.uint16).astype(np.uint32) << 16).view(np.float32)
    else:
        raise ValueError("%s: dtype %s" % (name, dt))
    return arr.reshape(meta["shape"])


class Case:
    """One golden case: the padded batch and the reference's outputs."""

    def __init__(self, gold_dir: str, rec: dict):
        self.name, self.rec = rec["name"], rec
        d = os.path.join(gold_dir, self.name)
        sh = rec["shapes"]

        def ld(key, dtype):
            return np.fromfile(os.path.join(d, key + ".bin"), dtype=dtype).reshape(sh[key])

        self.ids, self.att = ld("input_ids", np.int32), ld("attention_mask", np.int32)
        self.mpos, self.mmask = ld("marker_pos", np.int32), ld("marker_mask", np.int32)
        self.qtype, self.logits, self.act = ld("qtype", np.int32), ld("logits", np.float32), ld("act_logits", np.float32)
        self.layers = {k: ld(k, np.float32) for k in sh if k in ("emb", "final_norm", "head0", "head1")
                       or (k.startswith("enc") and k[3:].isdigit())}
        self.lens = self.att.sum(1).astype(np.int32)
        self.nm = self.mmask.sum(1).astype(np.int32)

    def abi_arrays(self):
        n = len(self.lens)
        ids = np.concatenate([self.ids[r, :self.lens[r]] for r in range(n)]).astype(np.int32)
        mk = np.concatenate([self.mpos[r, :self.nm[r]] for r in range(n)]).astype(np.int32)
        return self.lens, ids, self.nm.astype(np.int32), mk, self.qtype.astype(np.int32)

    def packed(self, key: str) -> np.ndarray:
        """The golden hidden state of every valid row, sequences back to back (the engine's layout)."""
        t = self.layers[key]
        return np.concatenate([t[r, :self.lens[r]] for r in range(len(self.lens))])

    def gathered(self, key: str) -> np.ndarray:
        """Rows of the engine's gathered last head layer: every question's markers, then first rows."""
        t = self.layers[key]
        n = len(self.lens)
        marks = [t[r, self.mpos[r, :self.nm[r]]] for r in range(n)]
        return np.concatenate(marks + [t[r, 0:1] for r in range(n)])


def rel(a, b) -> float:
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def layer_errors(case: Case, dump_dir: str, D: int, type_emb: Optional[np.ndarray]) -> Dict[str, float]:
    """max |a - b| / max |b| per hooked layer between the engine's dumps and the golden tensors."""
    def dump(name):
        return np.fromfile(os.path.join(dump_dir, name + ".bin"), np.float32).reshape(-1, D)

    out = {}
    for key in case.layers:
        if key == "head1":
            got, want = dump("head1"), case.gathered("head1")
        elif key == "final_norm":
            if type_emb is None:
                continue
            # the engine's "final" rows carry the question type's embedding, the hook's rows do not
            rows = np.concatenate([np.full(case.lens[r], case.qtype[r]) for r in range(len(case.lens))])
            got, want = dump("final") - type_emb[rows], case.packed("final_norm")
        else:
            got, want = dump(key), case.packed(key)
        out[key] = rel(got[:len(want)], want)
    return out


def api_errors(case: Case, logits: List[np.ndarray], cfg: dict) -> float:
    """Largest |probability difference| against the manifest's API answers (temperature-scaled)."""
    answers = case.rec.get("api", {}).get("answers", {})
    temps = cfg.get("temperature", [1.0, 1.0, 1.0])
    by_opt = cfg.get("temperature_by_options", {})
    worst = 0.0
    for (qid, ans), lg, qt in zip(answers.items(), logits, case.qtype):
        k = len(lg)
        size = "2" if k <= 2 else "3-5" if k <= 5 else "6-10" if k <= 10 else "11+"
        T = by_opt.get("%s:%s" % (QTYPE_NAMES[int(qt)], size), temps[int(qt)])
        p = _softmax(np.asarray(lg, np.float64) / T)
        if ans.get("type") == "noul":
            worst = max(worst, abs(round(float(p[1]), 4) - ans["noul"]))
        else:
            worst = max(worst, max(abs(round(float(v), 4) - w) for v, w in zip(p, ans["probabilities"].values())))
    return worst


def run(model_dir: str, gold_dir: str, precision: int = 0, devices: str = "", out=sys.stdout) -> dict:
    """Runs every case; returns {"rows", "fails", "worst_prob", "layers": {case: {layer: err}}, ...}."""
    from . import Engine

    with open(os.path.join(gold_dir, "manifest.json")) as f:
        manifest = json.load(f)
    with open(os.path.join(model_dir, "rl_agent_config.json")) as f:
        cfg = json.load(f)
    try:
        type_emb = read_tensor(os.path.join(model_dir, "model.safetensors"), "type_emb.weight")
    except (KeyError, ValueError, OSError):
        type_emb = None
    eng = Engine(model_dir, precision=precision, devices=devices)
    strict = precision == 1
    res = {"rows": 0, "fails": 0, "worst_prob": 0.0, "layers": {}, "worst_layer": 0.0, "worst_api": 0.0}
    print("\n%-24s %4s %5s %4s   %-11s %-11s %-11s  %s" % ("case", "row", "len", "K", "max|dlogit|", "max|dprob|",
                                                         "rel|dact|", "verdict"), file=out)
    dump_dir = tempfile.mkdtemp(prefix="laya_golden_")
    try:
        for pas in range(2):
            for rec in manifest["cases"]:
                case = Case(gold_dir, rec)
                lens, ids, nm, mk, qt = case.abi_arrays()
                seqs, marks, off, moff = [], [], 0, 0
                for r in range(len(lens)):
                    seqs.append(ids[off:off + lens[r]].tolist())
                    marks.append(mk[moff:moff + nm[r]].tolist())
                    off += lens[r]
                    moff += nm[r]
                if pas == 0:
                    eng.set_dump_dir(dump_dir)
                lo, ac, rc = eng.forward_batch_raw(seqs, marks, qt.tolist())
                if pas == 0:
                    eng.set_dump_dir(None)
                if rc != 0:
                    raise RuntimeError("%s: forward_batch returned %d" % (case.name, rc))
                logits, o = [], 0
                for r in range(len(lens)):
                    g, e = case.logits[r, :nm[r]], lo[o:o + nm[r]]
                    logits.append(e)
                    o += nm[r]
                    dl = float(np.abs(e - g).max())
                    dp = float(np.abs(_softmax(e) - _softmax(g)).max())
                    ga = case.act[r].astype(np.float64)
                    da = float((np.abs(ac[r] - ga) / np.maximum(1.0, np.abs(ga))).max())
                    ok = dp < 0.01 and da < 0.05 and (not strict or dp <= 1e-4)
                    res["rows"] += 1
                    res["fails"] += 0 if ok else 1
                    res["worst_prob"] = max(res["worst_prob"], dp)
                    print("%-24s %4d %5d %4d   %11.5f %11.6f %11.5f  %s" % (
                        case.name + (" [graph]" if pas else ""), r, lens[r], nm[r], dl, dp, da,
                        "PASS" if ok else "** FAIL **"), file=out)
                if pas == 0:
                    errs = {}
                    if case.layers:
                        D = next(iter(case.layers.values())).shape[-1]
                        errs = layer_errors(case, dump_dir, D, type_emb)
                    res["layers"][case.name] = errs
                    if errs:
                        k = max(errs, key=errs.get)
                        res["worst_layer"] = max(res["worst_layer"], errs[k])
                        bad = strict and errs[k] > 1e-3
                        res["fails"] += 1 if bad else 0
                        print("%-24s layers: worst %s %.2e%s" % (case.name, k, errs[k], "  ** FAIL **" if bad else ""),
                              file=out)
                    res["worst_api"] = max(res["worst_api"], api_errors(case, logits, cfg))
    finally:
        eng.close()
        shutil.rmtree(dump_dir, ignore_errors=True)
    print("\n%d/%d rows pass; worst probability delta = %.6f; worst layer error = %.2e; worst API "
          "probability delta = %.4f" % (res["rows"] - res["fails"], res["rows"], res["worst_prob"],
                                        res["worst_layer"], res["worst_api"]), file=out)
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Check the engine against a ref/gen_golden.py golden set.")
    ap.add_argument("model_dir")
    ap.add_argument("golden_dir")
    ap.add_argument("--precision", default="fp32parity", choices=["bf16", "fp32parity"])
    ap.add_argument("--devices", default="")
    args = ap.parse_args(argv)
    res = run(args.model_dir, args.golden_dir, 1 if args.precision == "fp32parity" else 0, args.devices)
    return 1 if res["fails"] else 0


if __name__ == "__main__":
    sys.exit(main())
