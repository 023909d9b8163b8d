"""Makes a fine-tuned checkpoint servable by this engine, or refuses it with the reasons.

    python -m layamd_b200.export BASE_DIR OUT_DIR

The counterpart of the reference's finetune/export.py:21-60. The trainer writes fp16 weights with a
re-saved tokenizer and encoder config; fine-tuning changes neither the tokenizer nor the encoder
shape, so the base checkpoint's ``tokenizer/`` and ``encoder/config.json`` are restored into OUT_DIR
(the files the engine and the request path were validated with) and the trainer's resume copy
``checkpoint_latest/`` is removed. Then OUT_DIR is checked against what the engine loads:
  - the same tensor names and shapes as the base's model.safetensors, in F16 / BF16 / F32;
  - the sequential option layout (the only one the request path builds);
  - max_len within the encoder's position table and the head depth of the base;
  - the model shape limits of this engine's kernels (head_dim 64, hidden size a multiple of 128 up to
    1024, GeGLU width a multiple of 64, 1 to 256 act outputs), which laya_create also enforces.
Only the safetensors headers are read; no weights are loaded and no GPU is used.
"""
import json
import os
import shutil
import struct
import sys
from typing import Dict, List

ENGINE_DTYPES = ("BF16", "F16", "F32")


def safetensors_header(path: str) -> Dict[str, dict]:
    """name -> {dtype, shape, data_offsets} from a safetensors file's JSON header."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
    header.pop("__metadata__", None)
    return header


def _json(path: str) -> dict:
    with open(path) as f:
        return json.load(f)


def restore_base_files(base: str, out: str):
    shutil.rmtree(os.path.join(out, "checkpoint_latest"), ignore_errors=True)
    for rel in ("tokenizer", os.path.join("encoder", "config.json")):
        src, dst = os.path.join(base, rel), os.path.join(out, rel)
        if os.path.isdir(src):
            shutil.rmtree(dst, ignore_errors=True)
            shutil.copytree(src, dst)
        elif os.path.exists(src):
            os.makedirs(os.path.dirname(dst), exist_ok=True)
            shutil.copy2(src, dst)


def check(base: str, out: str) -> List[str]:
    """Every reason OUT_DIR cannot be served (empty when it can)."""
    errors = []
    hb = safetensors_header(os.path.join(base, "model.safetensors"))
    ho = safetensors_header(os.path.join(out, "model.safetensors"))
    missing, extra = sorted(set(hb) - set(ho)), sorted(set(ho) - set(hb))
    if missing or extra:
        errors.append("tensor names differ from the base: missing %s, extra %s" % (missing[:5], extra[:5]))
    for name in sorted(set(hb) & set(ho)):
        if hb[name]["shape"] != ho[name]["shape"]:
            errors.append("%s: shape %s, base %s" % (name, ho[name]["shape"], hb[name]["shape"]))
    bad = sorted({t["dtype"] for t in ho.values()} - set(ENGINE_DTYPES))
    if bad:
        errors.append("dtypes %s are not loadable (engine takes %s)" % (bad, sorted(ENGINE_DTYPES)))

    cb = _json(os.path.join(base, "rl_agent_config.json"))
    co = _json(os.path.join(out, "rl_agent_config.json"))
    enc = _json(os.path.join(base, "encoder", "config.json"))
    if co.get("option_layout", "sequential") != "sequential":
        errors.append("option_layout %r: the engine implements the sequential layout only" % co["option_layout"])
    if co.get("max_len", 0) > enc.get("max_position_embeddings", 1 << 30):
        errors.append("max_len %s exceeds the encoder's %s positions" % (co["max_len"], enc["max_position_embeddings"]))
    if co.get("head_layers", cb.get("head_layers")) != cb.get("head_layers"):
        errors.append("head_layers changed from the base")

    d, heads = int(enc.get("hidden_size", 0)), int(enc.get("num_attention_heads", 1))
    inter = int(enc.get("intermediate_size", 0))
    n_act = len(co.get("act_costs", [])) + 1
    if heads <= 0 or d % heads != 0 or d // heads != 64:
        errors.append("head_dim %s: the attention kernels take 64" % (d / max(heads, 1)))
    if d % 128 != 0 or d > 1024:
        errors.append("hidden_size %d: the engine takes a multiple of 128 up to 1024" % d)
    if inter % 64 != 0:
        errors.append("intermediate_size %d: the engine takes a multiple of 64" % inter)
    if not 1 <= n_act <= 256:
        errors.append("%d act outputs: the engine takes 1 to 256" % n_act)
    if int(co.get("head_layers", 2)) < 1:
        errors.append("the decision head needs at least one layer")
    return errors


def summary(out: str) -> str:
    co = _json(os.path.join(out, "rl_agent_config.json"))
    ho = safetensors_header(os.path.join(out, "model.safetensors"))
    by_opt = co.get("temperature_by_options") or {}
    return "ok: %d tensors, max_len %s, head_max_len %s, temperatures %s%s" % (
        len(ho), co.get("max_len"), co.get("head_max_len"), co.get("temperature"),
        ", per-option-count buckets %s" % sorted(by_opt) if by_opt else "")


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) != 2:
        print(__doc__.strip().splitlines()[2].strip())
        return 2
    base, out = argv
    restore_base_files(base, out)
    errors = check(base, out)
    if errors:
        print("NOT servable by the engine:\n  " + "\n  ".join(errors))
        return 1
    print(summary(out))
    return 0


if __name__ == "__main__":
    sys.exit(main())
