"""Fine-tune export cases for the checkpoint validator (test infrastructure): each case is a trainer
output directory made from the tiny base checkpoint with one kind of change, plus the trainer's own
artefacts the export step must replace (a re-saved tokenizer, a resume copy)."""
import json
import os
import shutil

import numpy as np

from layamd_b200.synthetic import safetensors_io, synth

CASES = ("fp16", "names", "shape", "dtype", "layout", "maxlen", "headlayers", "several")


def _trainer_dir(base, out, weights, bf16_names=(), cfg_edit=None):
    os.makedirs(os.path.join(out, "encoder"), exist_ok=True)
    safetensors_io.write(os.path.join(out, "model.safetensors"), weights, bf16_names=bf16_names)
    with open(os.path.join(base, "rl_agent_config.json")) as f:
        cfg = json.load(f)
    if cfg_edit:
        cfg.update(cfg_edit)
    with open(os.path.join(out, "rl_agent_config.json"), "w") as f:
        json.dump(cfg, f)
    with open(os.path.join(out, "encoder", "config.json"), "w") as f:
        json.dump({"re-saved": True}, f)  # replaced by the base's
    os.makedirs(os.path.join(out, "tokenizer"), exist_ok=True)
    with open(os.path.join(out, "tokenizer", "tokenizer.json"), "w") as f:
        f.write("{}")  # replaced by the base's
    os.makedirs(os.path.join(out, "checkpoint_latest"), exist_ok=True)
    with open(os.path.join(out, "checkpoint_latest", "optimizer.pt"), "w") as f:
        f.write("x")


def fp16_weights(base):
    """The base weights as a trainer saves them: matrices in fp16, LayerNorm gains (1-D) in bf16."""
    w = safetensors_io.read(os.path.join(base, "model.safetensors"))
    out, bf16 = {}, []
    for k, v in w.items():
        if v.ndim >= 2:
            out[k] = v.astype(np.float16)
        else:
            out[k] = v
            bf16.append(k)
    return out, tuple(bf16)


def build(base, root, name):
    """Creates case `name` under root and returns its directory."""
    out = os.path.join(root, name)
    shutil.rmtree(out, ignore_errors=True)
    w, bf16 = fp16_weights(base)
    edit = None
    if name in ("names", "several"):
        w.pop("scorer.3.weight")
        w["extra.weight"] = np.zeros((4, 4), np.float16)
    if name == "shape":
        a = w["act_head.2.weight"]
        w["act_head.2.weight"] = np.concatenate([a, a[:1]], 0)
    if name == "dtype":
        w["type_emb.weight"] = np.zeros(w["type_emb.weight"].shape, np.int32)
    if name in ("layout", "several"):
        edit = {"option_layout": "interleaved"}
    if name == "maxlen":
        edit = {"max_len": 100000}
    if name == "headlayers":
        edit = {"head_layers": 3}
    _trainer_dir(base, out, w, bf16, edit)
    return out


def base_checkpoint():
    return synth.checkpoint("tiny", 0)
