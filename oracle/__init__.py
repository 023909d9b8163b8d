"""CPU oracle for the Laya encoder + decision-head forward pass -- TEST INFRASTRUCTURE ONLY.

Nothing in the engine (``layamd_b200``) imports, links or calls this package. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` / ``--impl reference`` leg) may
use it, and only as the checker or the timed CPU baseline, never as a compute path of the product.

Contents:
  model           numpy fp32 restatement of the reference forward pass (ref/rl_common.py
                  DecisionModel + transformers ModernBertModel), per-layer capture included
  ref_tools       builds the reference's own C++ host tools (src/bench_engine.cpp,
                  src/test_parity.cpp), unmodified, against this library into oracle/_ref

The seeded checkpoints and inputs it is run on come from ``layamd_b200.synthetic`` (input
generators, shared with the benchmarks; they compute nothing of the model).

Parity pin: ``model`` is checked against the reference's own PyTorch path (ref/rl_common.py with
the transformers ModernBertModel encoder) run in the build container on the same synthetic
checkpoints; the fixtures and the script that made them live in ``tests/golden/``.
"""
