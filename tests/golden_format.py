"""Writes a golden set in the reference's ref/gen_golden.py layout from the oracle (test
infrastructure): manifest.json plus, per case, the padded int32 inputs, fp32 logits / act logits and
the hooked hidden states, so that layamd_b200.golden_parity can be exercised without the reference's
real checkpoints."""
import json
import os

import numpy as np

from oracle import model as om
from layamd_b200.synthetic import synth

QT = ("choice", "score", "noul")


def cases(arch, seed=5):
    """A long single question, a yes/no, a 12-option choice and three questions of unequal lengths."""
    rng = np.random.default_rng(seed)

    def q(L, k, qt):
        ids = rng.integers(5, arch.vocab - 8, L).tolist()
        ids[0] = arch.cls_id
        marks = sorted(rng.choice(np.arange(1, L), k, replace=False).tolist())
        for m in marks:
            ids[m] = arch.mask_id
        return {"ids": ids, "markers": marks, "qtype": qt}

    L = arch.max_len
    return [("fill_ctx", [q(L, 4, 0)]), ("noul2_short", [q(20, 2, 2)]), ("choice12_long", [q(L - 10, 12, 0)]),
            ("multi_q", [q(L // 2, 3, 0), q(L - 3, 3, 1), q(40, 2, 2)])]


def write(model_dir, out_dir, seed=5):
    arch = synth.load_arch(model_dir)
    o = om.Oracle(synth.load_weights(model_dir), arch)
    with open(os.path.join(model_dir, "rl_agent_config.json")) as f:
        cfg = json.load(f)
    manifest = {"model_dir": model_dir, "cases": []}
    for name, qs in cases(arch, seed):
        n, Lmax, K = len(qs), max(len(x["ids"]) for x in qs), max(len(x["markers"]) for x in qs)
        ids = np.full((n, Lmax), arch.pad_id, np.int32)
        att = np.zeros((n, Lmax), np.int32)
        mpos = np.zeros((n, K), np.int32)
        mmask = np.zeros((n, K), np.int32)
        for r, x in enumerate(qs):
            ids[r, :len(x["ids"])] = x["ids"]
            att[r, :len(x["ids"])] = 1
            mpos[r, :len(x["markers"])] = x["markers"]
            mmask[r, :len(x["markers"])] = 1
        qt = np.array([x["qtype"] for x in qs], np.int32)
        lo, ac, caps = o.forward_batch(qs, capture=True)
        logits = np.zeros((n, K), np.float32)
        off = 0
        for r, x in enumerate(qs):
            logits[r, :len(x["markers"])] = lo[off:off + len(x["markers"])]
            off += len(x["markers"])
        layers = {}
        keys = ["emb"] + ["enc%d" % i for i in range(arch.layers)] + ["final_norm"] + \
               ["head%d" % j for j in range(arch.head_layers)]
        for k in keys:
            t = np.zeros((n, Lmax, arch.d), np.float32)
            for r, c in enumerate(caps):
                t[r, :len(qs[r]["ids"])] = c[k]
            layers[k] = t
        d = os.path.join(out_dir, name)
        os.makedirs(d, exist_ok=True)
        rec = {"name": name, "shapes": {}}
        for key, arr in [("input_ids", ids), ("attention_mask", att), ("marker_pos", mpos), ("marker_mask", mmask),
                         ("qtype", qt), ("logits", logits), ("act_logits", np.asarray(ac, np.float32))] + \
                list(layers.items()):
            arr = np.ascontiguousarray(arr)
            arr.tofile(os.path.join(d, key + ".bin"))
            rec["shapes"][key] = list(arr.shape)
        answers = {}
        for r, x in enumerate(qs):
            T = cfg.get("temperature", [1.0, 1.0, 1.0])[x["qtype"]]
            z = logits[r, :len(x["markers"])].astype(np.float64) / T
            p = np.exp(z - z.max())
            p /= p.sum()
            if x["qtype"] == 2:
                answers["q%d" % r] = {"type": "noul", "noul": round(float(p[1]), 4)}
            else:
                answers["q%d" % r] = {"type": QT[x["qtype"]],
                                      "probabilities": {"o%d" % i: round(float(v), 4) for i, v in enumerate(p)}}
        rec["api"] = {"answers": answers}
        rec["seq_lens"] = [len(x["ids"]) for x in qs]
        manifest["cases"].append(rec)
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        json.dump(manifest, f)
    return manifest
