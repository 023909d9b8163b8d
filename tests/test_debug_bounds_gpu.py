"""Debug bounds mode on a B200: the debug-bounds build (liblaya_b200_dbg.so, compiled with
-DLAYA_DEBUG_BOUNDS) gives exactly the normal build's results in both precisions, and a token id
planted one past the vocabulary after the host check (the build's LAYA_DEBUG_PLANT_ID test hook) is
caught by the embedding kernel's own bounds check on the device: the call returns -2 with code 40,
nothing is read out of range (the row it would read lies inside the table's allocation anyway), and
the next call succeeds. Each library runs in its own process."""
import json
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from layamd_b200 import LIB_PATH  # noqa: E402
from layamd_b200 import build as lb  # noqa: E402

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

RUN = textwrap.dedent("""
    import json, sys
    import numpy as np
    sys.path.insert(0, %(root)r)
    import layamd_b200
    L = layamd_b200.load_lib(%(lib)r)
    from tests.engine_helpers import Handle
    from layamd_b200.synthetic import synth, workloads
    ck = synth.checkpoint("tiny", 0)
    qs = workloads.mixed(synth.ARCHS["tiny"], 14, seed=5, kmax=6)
    out = {"build": int(L.laya_debug_bounds_build())}
    for prec in (0, 1):
        h = Handle(ck, prec, env=%(env)r)
        rcs = []
        for _ in range(2):
            rc, lo, ac = h.forward(qs)
            rcs.append(int(rc))
        h.close()
        out["rc%%d" %% prec] = rcs
        out["lo%%d" %% prec] = lo.tolist()
        out["ac%%d" %% prec] = ac.tolist()
    print("RESULT " + json.dumps(out), flush=True)
""")


def run(lib, env=None):
    env = dict(env or {})
    env.setdefault("LAYA_MAX_TOKENS", "4096")
    r = subprocess.run([sys.executable, "-c", RUN % {"root": ROOT, "lib": lib, "env": env}], capture_output=True,
                       text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stdout + r.stderr
    line = [x for x in r.stdout.splitlines() if x.startswith("RESULT ")][-1]
    return json.loads(line[7:]), r.stderr


@pytest.fixture(scope="module")
def normal():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    if not os.path.exists(lb.LIB_DBG):
        pytest.fail("debug bounds build missing: python -m layamd_b200.build --debug-bounds")
    return run(LIB_PATH)[0]


def test_debug_build_matches_normal_build(normal):
    dbg, _ = run(lb.LIB_DBG)
    assert normal["build"] == 0 and dbg["build"] == 1
    for prec in (0, 1):
        assert normal["rc%d" % prec] == [0, 0] and dbg["rc%d" % prec] == [0, 0]
        assert np.array_equal(np.asarray(dbg["lo%d" % prec]), np.asarray(normal["lo%d" % prec]))
        assert np.array_equal(np.asarray(dbg["ac%d" % prec]), np.asarray(normal["ac%d" % prec]))


def test_planted_token_id_is_caught_on_the_device(normal):
    dbg, err = run(lb.LIB_DBG, {"LAYA_DEBUG_PLANT_ID": "1"})
    for prec in (0, 1):  # each handle's first pass carries the planted id; the second call is clean
        assert dbg["rc%d" % prec] == [-2, 0], dbg["rc%d" % prec]
        assert np.array_equal(np.asarray(dbg["lo%d" % prec]), np.asarray(normal["lo%d" % prec]))
    assert "kernel code 40" in err
