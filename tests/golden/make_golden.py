"""Generates the golden fixtures in tests/golden/ by running the reference's own PyTorch path.

Run in the build container (it imports the reference's ref/rl_common.py from the reference checkout,
LAYA_REFERENCE or a directory named "reference" beside the repository, plus the installed transformers
ModernBertModel; neither exists on the GPU boxes, which only read the committed .npz files):

    python tests/golden/make_golden.py              # every fixture
    python tests/golden/make_golden.py --configs    # only the C3 / C4 ones
    python tests/golden/make_golden.py --c2         # only the C2 batch's logits
    python tests/golden/make_golden.py --c3c4       # only the whole C3 and C4 batches' logits
    python tests/golden/make_golden.py --seq512     # only the fixed-length 512 batch's logits

What it does, following ref/gen_golden.py:51-105 of the reference:
  1. builds each synthetic checkpoint with layamd_b200.synthetic.synth (seeded init rule) and checks that the
     reference DecisionModel (ref/rl_common.py:127-134 build_model, attn_implementation="sdpa") has
     exactly the tensor names, order and shapes the generator writes, then loads it strict=True;
  2. runs the model in fp32 on CPU on each case as ONE padded batch (collate_items,
     ref/rl_common.py:265-293), with forward hooks on the embeddings, every encoder layer, the final
     norm and every head layer (ref/gen_golden.py:58-71);
  3. saves logits, act logits, inputs and the hooked activations (full tensors for the tiny model;
     row norms plus sampled rows for the ModernBERT-large C1 case, which would be 70 MB in full).
A fingerprint of every generated weight tensor is stored too, so the GPU-side tests can check that
their regenerated checkpoint is the one the fixtures were made from.
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from layamd_b200.synthetic import synth, workloads  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
from oracle.ref_tools import reference_root  # noqa: E402

REF = reference_root()


def fingerprint(weights):
    """name -> (sum, sum of squares, first element) in float64: cheap, order-sensitive identity."""
    fp = {}
    for k, v in weights.items():
        v64 = np.asarray(v, dtype=np.float64).ravel()
        fp[k] = np.array([v64.sum(), (v64 * v64).sum(), v64[0]])
    return fp


def reference_model(ckpt):
    import torch
    sys.path.insert(0, os.path.join(REF, "ref"))
    import rl_common  # the reference's upstream model file, unmodified
    import json
    cfg = json.load(open(os.path.join(ckpt, "rl_agent_config.json")))
    model = rl_common.build_model(cfg, encoder_dir=os.path.join(ckpt, "encoder"))
    sd = model.state_dict()
    specs = synth.param_specs(synth.load_arch(ckpt))
    names = [n for n, _, _ in specs]
    assert list(sd.keys()) == names, "state_dict order differs from layamd_b200.synthetic.synth.param_specs"
    for n, shape, _ in specs:
        assert tuple(sd[n].shape) == tuple(shape), (n, sd[n].shape, shape)
    w = synth.load_weights(ckpt)
    model.load_state_dict({k: torch.from_numpy(np.array(v)) for k, v in w.items()}, strict=True)
    model.float().eval()
    return model, rl_common, w


def run_reference(model, rl_common, arch, questions):
    import torch
    acts = {}
    hooks = []

    def cap(name):
        def fn(mod, inp, out):
            t = out[0] if isinstance(out, tuple) else out
            if torch.is_tensor(t):
                acts[name] = t.detach().float().cpu().numpy()
        return fn

    enc = model.encoder
    hooks.append(enc.embeddings.register_forward_hook(cap("emb")))
    for i, lyr in enumerate(enc.layers):
        hooks.append(lyr.register_forward_hook(cap("enc%d" % i)))
    hooks.append(enc.final_norm.register_forward_hook(cap("final_norm")))
    for j, lyr in enumerate(model.head.layers):
        hooks.append(lyr.register_forward_hook(cap("head%d" % j)))
    items = [{"ids": q["ids"], "markers": q["markers"], "qtype": q["qtype"], "target": [0.0] * len(q["markers"]),
              "label": -1, "episode": 0, "ep_step": 0, "ep_len": 1, "src": "golden"} for q in questions]
    b = rl_common.collate_items([items], arch.pad_id)
    with torch.no_grad():
        logits, act = model(b["input_ids"], b["attention_mask"], b["marker_pos"], b["marker_mask"], b["qtype"])
    for h in hooks:
        h.remove()
    return logits.numpy(), act.numpy(), acts, b


def save_case(path, questions, logits, act, acts, full, sample_rows=None):
    out = {}
    lens = [len(q["ids"]) for q in questions]
    nm = [len(q["markers"]) for q in questions]
    lens_, ids, nmark, markers, qtypes = workloads.flatten(questions)
    out.update(lens=lens_, ids=ids, nmark=nmark, markers=markers, qtypes=qtypes)
    out["logits"] = np.concatenate([logits[r, :nm[r]] for r in range(len(questions))]).astype(np.float32)
    out["act"] = act.astype(np.float32)
    for k, v in acts.items():
        rows = [v[r, :lens[r]] for r in range(len(questions))]
        if full:
            out["t_" + k] = np.concatenate(rows).astype(np.float32)
        else:
            out["n_" + k] = np.concatenate([np.linalg.norm(x, axis=-1) for x in rows]).astype(np.float32)
            out["s_" + k] = np.stack([rows[0][i] for i in sample_rows]).astype(np.float32)
    if sample_rows is not None:
        out["sample_rows"] = np.array(sample_rows, np.int32)
    np.savez_compressed(path, **out)


def main():
    import torch
    torch.set_grad_enabled(False)
    torch.set_num_threads(os.cpu_count() or 8)
    # tiny model: three cases (mixed batch with every qtype and 1..6 options, a one-option question,
    # a full-context question), full per-layer tensors
    a = synth.ARCHS["tiny"]
    ck = synth.checkpoint("tiny", 0)
    model, rl, w = reference_model(ck)
    np.savez_compressed(os.path.join(HERE, "tiny_weights_fp.npz"), **fingerprint(w))
    cases = {
        "tiny_mixed": workloads.mixed(a, 5, seed=21, kmax=6),
        # a one-option question batched with a 3-option one: the reference pads its logits with
        # -1e4 (ref/rl_common.py:115), so top2 = 0 for it (topk(2) needs a 2-wide batch)
        "tiny_k1": [workloads._question(np.random.default_rng(22), 40, 1, 0, a),
                    workloads._question(np.random.default_rng(23), 70, 3, 1, a)],
        "tiny_full": [workloads._question(np.random.default_rng(24), a.max_len, 4, 1, a)],
    }
    for name, qs in cases.items():
        lo, ac, acts, b = run_reference(model, rl, a, qs)
        save_case(os.path.join(HERE, name + ".npz"), qs, lo, ac, acts, full=True)
        print("[golden] %-10s lens=%s" % (name, [len(q["ids"]) for q in qs]), flush=True)
    # ModernBERT-large C1: batch 1, seq 512, 3-option choice
    a = synth.ARCHS["large"]
    ck = synth.checkpoint("large", 0)
    model, rl, w = reference_model(ck)
    np.savez_compressed(os.path.join(HERE, "large_weights_fp.npz"), **fingerprint(w))
    qs = workloads.c1(a)
    lo, ac, acts, b = run_reference(model, rl, a, qs)
    save_case(os.path.join(HERE, "large_c1.npz"), qs, lo, ac, acts, full=False,
              sample_rows=[0, 1, 16, 24, 32, 100, 257, 511])
    print("[golden] large_c1 logits=%s act=%s" % (lo[0], ac[0]), flush=True)
    # ModernBERT-large, 3 questions of unequal length in one padded batch (reference multi_q shape)
    rng = np.random.default_rng(5)
    qs = [workloads._question(rng, 218, 5, 1, a), workloads._question(rng, 199, 3, 0, a),
          workloads._question(rng, 215, 2, 2, a)]
    lo, ac, acts, b = run_reference(model, rl, a, qs)
    save_case(os.path.join(HERE, "large_multi.npz"), qs, lo, ac, acts, full=False, sample_rows=[0, 1, 2])
    print("[golden] large_multi lens=%s" % [len(q["ids"]) for q in qs], flush=True)
    del model
    configs()
    c2_batch()
    c3c4_batches()
    seq512_batch()


def configs():
    """The other benchmark configurations: mmBERT-base (C3: vocabulary 256,000, pad id 0, 22 layers,
    d 768) and ModernBERT-large at context 1024 (C4: RoPE positions 512-1023, global attention over
    more than 512 keys), each with a question longer than 900 tokens in a padded batch."""
    # C3: token ids over the whole vocabulary (pad id 0 included inside a sequence, as C3 draws them)
    a = synth.ARCHS["base"]
    ck = synth.checkpoint("base", 0)
    model, rl, w = reference_model(ck)
    np.savez_compressed(os.path.join(HERE, "base_weights_fp.npz"), **fingerprint(w))
    rng = np.random.default_rng(31)
    qs = [workloads._question(rng, 987, 3, 0, a, id_lo=0), workloads._question(rng, 301, 3, 0, a, id_lo=0)]
    lo, ac, acts, b = run_reference(model, rl, a, qs)
    save_case(os.path.join(HERE, "base_c3.npz"), qs, lo, ac, acts, full=False,
              sample_rows=[0, 1, 2, 511, 512, 700, 900, 986])
    print("[golden] base_c3 lens=%s" % [len(q["ids"]) for q in qs], flush=True)
    del model
    # C4: the ModernBERT-large weights with a context-1024 agent config; all three question types
    a = synth.ARCHS["large1024"]
    ck = synth.checkpoint("large1024", 0)
    model, rl, w = reference_model(ck)
    np.savez_compressed(os.path.join(HERE, "large1024_weights_fp.npz"), **fingerprint(w))
    rng = np.random.default_rng(41)
    qs = [workloads._question(rng, 1021, 4, 1, a), workloads._question(rng, 377, 2, 2, a),
          workloads._question(rng, 733, 6, 0, a)]
    lo, ac, acts, b = run_reference(model, rl, a, qs)
    save_case(os.path.join(HERE, "large1024_c4.npz"), qs, lo, ac, acts, full=False,
              sample_rows=[0, 1, 17, 511, 512, 513, 800, 1020])
    print("[golden] large1024_c4 lens=%s" % [len(q["ids"]) for q in qs], flush=True)


def c2_batch():
    """Logits and act logits of the reference for the whole C2 benchmark batch (ModernBERT-large, 64
    states x 3 questions, seed 1), run in length-sorted padded batches of 16 as predict_items does
    (ref/rl_common.py:370-408); no hooks."""
    batch_logits("large", workloads.c2(synth.ARCHS["large"], seed=1), "large_c2_logits.npz")


def c3c4_batches():
    """The same for the whole C3 batch (mmBERT-base, 128 questions, L ~ U[64,1024], seed 3) and the
    whole C4 batch (ModernBERT-large at context 1024, 256 questions, L log-uniform in [128,1024],
    seed 4), the batches workload_bench serves."""
    batch_logits("base", workloads.c3(synth.ARCHS["base"], seed=3), "base_c3_logits.npz")
    batch_logits("large1024", workloads.c4(synth.ARCHS["large1024"], seed=4), "large1024_c4_logits.npz")


def seq512_batch():
    """The same for the bench's fixed-length batch (128 choice questions of exactly 512 tokens with 3
    options, seed 5)."""
    batch_logits("large", workloads.seq512(synth.ARCHS["large"], seed=5), "large_seq512_logits.npz")


def batch_logits(arch_name, qs, out_name):
    a = synth.ARCHS[arch_name]
    ck = synth.checkpoint(arch_name, 0)
    model, rl, w = reference_model(ck)
    order = sorted(range(len(qs)), key=lambda i: len(qs[i]["ids"]))
    logits = [None] * len(qs)
    act = np.zeros((len(qs), a.n_act), np.float32)
    for s in range(0, len(order), 16):
        idx = order[s:s + 16]
        lo, ac, _, _ = run_reference(model, rl, a, [qs[i] for i in idx])
        for r, i in enumerate(idx):
            logits[i] = lo[r, :len(qs[i]["markers"])]
            act[i] = ac[r]
    lens, ids, nmark, markers, qtypes = workloads.flatten(qs)
    np.savez_compressed(os.path.join(HERE, out_name), lens=lens, nmark=nmark, qtypes=qtypes,
                        markers=markers, ids_sum=np.int64(ids.astype(np.int64).sum()),
                        logits=np.concatenate(logits).astype(np.float32), act=act)
    print("[golden] %s: %d questions, %d tokens" % (out_name, len(qs), int(lens.sum())), flush=True)


if __name__ == "__main__":
    steps = {"--configs": configs, "--c2": c2_batch, "--c3c4": c3c4_batches, "--seq512": seq512_batch}
    if len(sys.argv) == 2 and sys.argv[1] in steps:
        import torch
        torch.set_grad_enabled(False)
        torch.set_num_threads(os.cpu_count() or 8)
        steps[sys.argv[1]]()
    else:
        main()
