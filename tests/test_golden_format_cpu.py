"""The golden-set reader of layamd_b200.golden_parity on a set written in the reference's layout:
inputs come back as the ABI arrays, hidden states in the engine's packed and gathered row orders."""
import json
import os

import numpy as np

from layamd_b200 import golden_parity as G
from layamd_b200.synthetic import synth
from tests import golden_format


def test_reader_round_trip(tmp_path):
    ck = synth.checkpoint("tiny", 0)
    man = golden_format.write(ck, str(tmp_path))
    arch = synth.load_arch(ck)
    qs_all = dict(golden_format.cases(arch))
    assert [c["name"] for c in json.load(open(os.path.join(tmp_path, "manifest.json")))["cases"]] == list(qs_all)
    for rec in man["cases"]:
        c = G.Case(str(tmp_path), rec)
        qs = qs_all[rec["name"]]
        lens, ids, nm, mk, qt = c.abi_arrays()
        assert lens.tolist() == [len(q["ids"]) for q in qs]
        assert ids.tolist() == [t for q in qs for t in q["ids"]]
        assert mk.tolist() == [m for q in qs for m in q["markers"]] and nm.tolist() == [len(q["markers"]) for q in qs]
        assert qt.tolist() == [q["qtype"] for q in qs]
        assert c.packed("enc0").shape == (sum(lens), arch.d)
        assert c.gathered("head1").shape == (sum(nm) + len(qs), arch.d)
        # the first gathered row is the first question's first marker
        assert np.array_equal(c.gathered("head1")[0], c.layers["head1"][0, qs[0]["markers"][0]])
    te = G.read_tensor(os.path.join(ck, "model.safetensors"), "type_emb.weight")
    assert te.shape == (3, arch.d) and te.dtype == np.float32
