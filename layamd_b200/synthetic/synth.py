"""Seeded random-init Laya checkpoints in the reference's on-disk layout, for the tests and the
benchmarks (no real checkpoint is available to them).

A checkpoint directory holds what the reference engine loads (src/engine.hip:140-176,
src/laya.cpp:5-41): ``model.safetensors`` with the reference tensor names, ``encoder/config.json``
(a ModernBertConfig, including ``layer_types`` and ``rope_parameters``) and ``rl_agent_config.json``.

Init rule (the benchmark configurations' "seed 0, N(0,0.02)"): one ``torch.Generator`` seeded with
`seed`; tensors drawn in the reference ``DecisionModel.state_dict()`` order (ref/rl_common.py:81-97
with transformers' ModernBertModel as encoder): every weight matrix, embedding and bias
~ N(0, 0.02); every LayerNorm gain = 1 + N(0, 0.02); the ``temperature`` buffer = ones. The name
order is checked against the real reference model by tests/golden/make_golden.py.
"""
import hashlib
import json
import os
from dataclasses import asdict, dataclass, field
from typing import Dict, List

import numpy as np

from . import safetensors_io


@dataclass
class Arch:
    name: str
    vocab: int
    d: int
    heads: int
    inter: int
    layers: int
    global_every: int = 3
    local_attention: int = 128
    theta_global: float = 160000.0
    theta_local: float = 10000.0
    eps: float = 1e-5
    pad_id: int = 50283
    cls_id: int = 50281
    sep_id: int = 50282
    mask_id: int = 50284
    max_len: int = 512
    head_max_len: int = 192
    head_layers: int = 2
    n_act: int = 2
    temperature: List[float] = field(default_factory=lambda: [1.0, 1.0, 1.0])

    def layer_types(self):
        return ["full_attention" if i % self.global_every == 0 else "sliding_attention" for i in range(self.layers)]


# ModernBERT-large (laya-en) and mmBERT-base (laya-multi) shapes, docs/architecture.md of the
# reference; "tiny" is a 4-layer model of the same structure for fast parity cases.
ARCHS: Dict[str, Arch] = {
    "large": Arch("large", 50368, 1024, 16, 2624, 28),
    "large1024": Arch("large1024", 50368, 1024, 16, 2624, 28, max_len=1024, head_max_len=256),
    "base": Arch("base", 256000, 768, 12, 1152, 22, pad_id=0, cls_id=2, sep_id=1, mask_id=4, max_len=1024,
                 head_max_len=256),
    "tiny": Arch("tiny", 1000, 128, 2, 192, 4, local_attention=16, pad_id=999, cls_id=997, sep_id=998,
                 mask_id=996, max_len=128, head_max_len=48, n_act=3, temperature=[0.7, 1.3, 2.0]),
}
# architectures that share one weight file (same tensors, different agent config)
WEIGHTS_OF = {"large1024": "large"}


def param_specs(a: Arch):
    """(name, shape, kind) in DecisionModel.state_dict() order; kind: 'w' N(0,.02), 'g' 1+N(0,.02), 'one'."""
    D, I, V = a.d, a.inter, a.vocab
    # DecisionModel's own buffer comes before its submodules in state_dict()
    s = [("temperature", (3,), "one"), ("encoder.embeddings.tok_embeddings.weight", (V, D), "w"),
         ("encoder.embeddings.norm.weight", (D,), "g")]
    for i in range(a.layers):
        p = "encoder.layers.%d." % i
        if i > 0:
            s.append((p + "attn_norm.weight", (D,), "g"))
        s += [(p + "attn.Wqkv.weight", (3 * D, D), "w"), (p + "attn.Wo.weight", (D, D), "w"),
              (p + "mlp_norm.weight", (D,), "g"), (p + "mlp.Wi.weight", (2 * I, D), "w"),
              (p + "mlp.Wo.weight", (D, I), "w")]
    s.append(("encoder.final_norm.weight", (D,), "g"))
    for j in range(a.head_layers):
        p = "head.layers.%d." % j
        s += [(p + "self_attn.in_proj_weight", (3 * D, D), "w"), (p + "self_attn.in_proj_bias", (3 * D,), "w"),
              (p + "self_attn.out_proj.weight", (D, D), "w"), (p + "self_attn.out_proj.bias", (D,), "w"),
              (p + "linear1.weight", (4 * D, D), "w"), (p + "linear1.bias", (4 * D,), "w"),
              (p + "linear2.weight", (D, 4 * D), "w"), (p + "linear2.bias", (D,), "w"),
              (p + "norm1.weight", (D,), "g"), (p + "norm1.bias", (D,), "w"),
              (p + "norm2.weight", (D,), "g"), (p + "norm2.bias", (D,), "w")]
    s += [("type_emb.weight", (3, D), "w"), ("scorer.0.weight", (D,), "g"), ("scorer.0.bias", (D,), "w"),
          ("scorer.1.weight", (D, D), "w"), ("scorer.1.bias", (D,), "w"), ("scorer.3.weight", (1, D), "w"),
          ("scorer.3.bias", (1,), "w"), ("act_head.0.weight", (256, D + 4), "w"), ("act_head.0.bias", (256,), "w"),
          ("act_head.2.weight", (a.n_act, 256), "w"), ("act_head.2.bias", (a.n_act,), "w")]
    return s


def generate_tensors(a: Arch, seed: int = 0):
    """Ordered dict name -> fp32 numpy array following the init rule above."""
    import torch
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape, kind in param_specs(a):
        if kind == "one":
            t = torch.ones(shape)
        else:
            t = torch.randn(shape, generator=g, dtype=torch.float32) * 0.02
            if kind == "g":
                t = t + 1.0
        out[name] = t.numpy()
    return out


def encoder_config(a: Arch):
    return {
        "architectures": ["ModernBertModel"], "model_type": "modernbert", "vocab_size": a.vocab,
        "hidden_size": a.d, "intermediate_size": a.inter, "num_hidden_layers": a.layers,
        "num_attention_heads": a.heads, "hidden_activation": "gelu", "max_position_embeddings": max(a.max_len, 512),
        "norm_eps": a.eps, "norm_bias": False, "pad_token_id": a.pad_id, "cls_token_id": a.cls_id,
        "sep_token_id": a.sep_id, "bos_token_id": a.cls_id, "eos_token_id": a.sep_id, "mask_token_id": a.mask_id,
        "attention_bias": False, "mlp_bias": False, "global_attn_every_n_layers": a.global_every,
        "local_attention": a.local_attention, "layer_types": a.layer_types(),
        "rope_parameters": {"full_attention": {"rope_type": "default", "rope_theta": a.theta_global},
                            "sliding_attention": {"rope_type": "default", "rope_theta": a.theta_local}},
        "attention_dropout": 0.0, "embedding_dropout": 0.0, "mlp_dropout": 0.0,
    }


def agent_config(a: Arch):
    return {"encoder": "synthetic", "max_len": a.max_len, "head_max_len": a.head_max_len,
            "head_layers": a.head_layers, "act_costs": [0.01] * (a.n_act - 1), "temperature": list(a.temperature),
            "amp_dtype": "bf16"}


# ---- synthetic tokenizer (the request path's tests and benchmark; real checkpoints ship their own).
# A word-level vocabulary over the words the request layout itself writes ("choice question:",
# "level 0:", the yes/no option texts, JSON punctuation runs) plus everyday words and numbers, then
# filler tokens "t<id>" up to the model's vocabulary size; [MASK] / [CLS] / [SEP] / [PAD] sit at the
# architecture's special ids and [UNK] at the lowest free id. Pre-tokenisation splits on whitespace
# and punctuation runs, so one word is one token and sequence lengths are easy to control.
_TOKEN_WORDS = (
    "choice score noul question level false true no yes the statement does not hold holds is a an of to in it and "
    "or for on with as at by this that be are was were has have had will would can could should may might what which "
    "who how when where why user agent state goal task step action next best open closed door light room key box item "
    "table chair left right up down move pick drop wait go stop done ready safe unsafe good bad high low red green blue "
    "answer response correct wrong helpful relevant quality rate reached found empty full true_ false_ "
    "0 1 2 3 4 5 6 7 8 9 10 11 12 13 14 15 16 17 18 19 20 100 1000").split() + [
    ":", ",", ".", "?", "!", "-", "(", ")", "/", "'", '"', "{", "}", "[", "]", '{"', '":', '",', '"}', '"]', '["',
    '":"', '","', '"},', "},", "}}", "]}", "\\"]


def tokenizer_vocab(a: Arch) -> Dict[str, int]:
    special = {"[MASK]": a.mask_id, "[CLS]": a.cls_id, "[SEP]": a.sep_id, "[PAD]": a.pad_id}
    taken = set(special.values())
    words = ["[UNK]"] + list(dict.fromkeys(_TOKEN_WORDS))
    vocab = dict(special)
    i = 0
    for idx in range(a.vocab):  # dense ids: the tokenizers library warns about holes
        if idx in taken:
            continue
        vocab[words[i] if i < len(words) else "t%d" % idx] = idx
        i += 1
    return vocab


def write_tokenizer(out_dir: str, a: Arch):
    """Writes tokenizer.json and tokenizer_config.json (the files the request path loads) into out_dir."""
    from tokenizers import Tokenizer, models, pre_tokenizers

    os.makedirs(out_dir, exist_ok=True)
    t = Tokenizer(models.WordLevel(vocab=tokenizer_vocab(a), unk_token="[UNK]"))
    t.pre_tokenizer = pre_tokenizers.Whitespace()
    t.add_special_tokens(["[MASK]", "[CLS]", "[SEP]", "[PAD]"])
    tmp = os.path.join(out_dir, "tokenizer.json.tmp")
    t.save(tmp)
    os.replace(tmp, os.path.join(out_dir, "tokenizer.json"))
    with open(os.path.join(out_dir, "tokenizer_config.json"), "w") as f:
        json.dump({"mask_token": "[MASK]", "cls_token": "[CLS]", "sep_token": "[SEP]", "pad_token": "[PAD]"}, f)


def default_root():
    return os.environ.get("LAYA_SYNTH_DIR", "/tmp/laya_synth")


def checkpoint(arch: str, seed: int = 0, root: str = None) -> str:
    """Returns the directory of the seeded checkpoint for `arch`, generating it on first use."""
    a = ARCHS[arch]
    root = root or default_root()
    key = hashlib.sha1(json.dumps([asdict(a), seed, 3]).encode()).hexdigest()[:10]
    d = os.path.join(root, "%s-s%d-%s" % (arch, seed, key))
    done = os.path.join(d, ".complete")
    if os.path.exists(done):
        if not os.path.exists(os.path.join(d, "tokenizer", "tokenizer.json")):
            write_tokenizer(os.path.join(d, "tokenizer"), a)
        return d
    os.makedirs(os.path.join(d, "encoder"), exist_ok=True)
    wsrc = WEIGHTS_OF.get(arch)
    st = os.path.join(d, "model.safetensors")
    if wsrc:
        src = os.path.join(checkpoint(wsrc, seed, root), "model.safetensors")
        if os.path.lexists(st):
            os.remove(st)
        os.symlink(src, st)
    else:
        tmp = st + ".tmp"
        safetensors_io.write(tmp, generate_tensors(a, seed))
        os.replace(tmp, st)
    with open(os.path.join(d, "encoder", "config.json"), "w") as f:
        json.dump(encoder_config(a), f, indent=1)
    with open(os.path.join(d, "rl_agent_config.json"), "w") as f:
        json.dump(agent_config(a), f, indent=1)
    write_tokenizer(os.path.join(d, "tokenizer"), a)
    open(done, "w").close()
    return d


def load_weights(ckpt_dir: str):
    return safetensors_io.read(os.path.join(ckpt_dir, "model.safetensors"))


def load_arch(ckpt_dir: str) -> Arch:
    """Architecture of a checkpoint directory from its two config files."""
    with open(os.path.join(ckpt_dir, "encoder", "config.json")) as f:
        e = json.load(f)
    with open(os.path.join(ckpt_dir, "rl_agent_config.json")) as f:
        g = json.load(f)
    every = e.get("global_attn_every_n_layers", 3)
    a = Arch("custom", e["vocab_size"], e["hidden_size"], e["num_attention_heads"], e["intermediate_size"],
             e["num_hidden_layers"], global_every=every, local_attention=e.get("local_attention", 128),
             eps=e.get("norm_eps", 1e-5), pad_id=e.get("pad_token_id", 50283), cls_id=e.get("cls_token_id", 50281),
             sep_id=e.get("sep_token_id", 50282), mask_id=e.get("mask_token_id", 50284),
             max_len=g.get("max_len", 512), head_max_len=g.get("head_max_len", 192),
             head_layers=g.get("head_layers", 2), n_act=len(g.get("act_costs", [0])) + 1,
             temperature=g.get("temperature", [1.0, 1.0, 1.0]))
    rp = e.get("rope_parameters", {})
    a.theta_global = float(rp.get("full_attention", {}).get("rope_theta", 160000.0))
    a.theta_local = float(rp.get("sliding_attention", {}).get("rope_theta", 10000.0))
    lt = e.get("layer_types")
    a._layer_types = lt if lt else a.layer_types()
    return a
