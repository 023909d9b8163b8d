"""Laya B200 engine: host-side Python binding of ``liblaya_b200.so``.

The product is the C ABI in ``include/laya_api.h`` (the reference's ``src/laya_api.h`` plus
additions). This module is the Python mirror of the reference's ctypes binding
(mauimauer/layamd server/laya_server.py:18-50, class ``Engine``): same method names, argument
meaning and error behaviour, so callers written against the reference server run unchanged. There is
no Python or CPU compute path: if the shared library is missing the import of ``load_lib`` fails.
"""
import ctypes
import itertools
import os
from array import array
from typing import List, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblaya_b200.so")

_IP = ctypes.POINTER(ctypes.c_int)
_FP = ctypes.POINTER(ctypes.c_float)
_lib = None

PRECISION_BF16 = 0
PRECISION_FP32_PARITY = 1


def load_lib(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads the engine library once and declares every exported signature. Raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise RuntimeError("liblaya_b200.so not built (run python -m layamd_b200.build): %s" % path)
    L = ctypes.CDLL(path)
    vp, i, f, d = ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_double
    sig = {
        "laya_create": (vp, [ctypes.c_char_p]),
        "laya_forward_batch": (i, [vp, i, _IP, _IP, _IP, _IP, _IP, _FP, _FP]),
        "laya_forward": (None, [vp, _IP, i, i, _IP, i, i, _FP, _FP]),
        "laya_n_act": (i, [vp]),
        "laya_max_len": (i, [vp]),
        "laya_max_markers": (i, [vp]),
        "laya_temperature": (f, [vp, i]),
        "laya_prof_report": (None, [vp, i]),
        "laya_prof_reset": (None, [vp]),
        "laya_tune_all": (None, [vp]),
        "laya_destroy": (None, [vp]),
        "laya_create_ex": (vp, [ctypes.c_char_p, i, ctypes.c_char_p]),
        "laya_num_devices": (i, [vp]),
        "laya_prof_enable": (None, [vp, i]),
        "laya_prof_get": (i, [vp, ctypes.c_char_p, ctypes.POINTER(d), ctypes.POINTER(ctypes.c_longlong)]),
        "laya_plan_passes": (i, [vp, i, _IP, _IP, _IP, i, _IP, _IP, _IP]),
        "laya_plan_passes_cfg": (i, [i, i, i, i, _IP, _IP, _IP, i, _IP, _IP, _IP]),
        "laya_shard_plan": (i, [i, i, _IP, _IP, i, i, i, i, i, _IP]),
        "laya_stage": (i, [vp, i, _IP, _IP, _IP, _IP, _IP]),
        "laya_replay": (i, [vp, i, ctypes.POINTER(d)]),
        "laya_replay_profiled": (i, [vp, i]),
        "laya_plan_gemm": (i, [i, i, i, i, i, i, i, _IP, _IP]),
        "laya_b200_watchdog_selftest": (i, [i, ctypes.POINTER(i), ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(f)]),
        "laya_staged_results": (i, [vp, _FP, _FP]),
        "laya_set_dump_dir": (i, [vp, ctypes.c_char_p]),
        "laya_io_stats": (i, [vp, ctypes.POINTER(ctypes.c_longlong), ctypes.POINTER(ctypes.c_longlong),
                              ctypes.POINTER(ctypes.c_longlong), i]),
        "laya_b200_gemm": (i, [vp, vp, vp, vp, vp, i, i, i, i, i, i, i, i, vp, vp, vp, i, i, vp, i]),
        "laya_b200_gemm_splitk": (i, [vp, vp, vp, vp, vp, i, i, i, i, i, i, i, i, vp, vp, vp, i, i, i, vp, i]),
        "laya_b200_attention": (i, [vp, vp, i, i, _IP, i, i, i, vp, i]),
        "laya_b200_gemm_splitk_noalloc": (i, [vp, vp, vp, vp, vp, i, i, i, i, i, i, i, i, vp, vp, vp, i, i, i, vp, i]),
        "laya_b200_kernel_error": (i, [i]),
        "laya_pack_check": (i, [i, i, i, i, i, i, _IP, _IP, _IP, _IP, _IP, i]),
        "laya_debug_bounds_build": (i, []),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _ia(a) -> ctypes.Array:
    a = np.ascontiguousarray(np.asarray(a, dtype=np.int32))
    return a, a.ctypes.data_as(_IP)


class Engine:
    """One engine handle. Mirrors the reference's ctypes ``Engine`` (server/laya_server.py:18-50)."""

    def __init__(self, model_dir: str, precision: int = PRECISION_BF16, devices: str = ""):
        self.lib = L = load_lib()
        self.h = L.laya_create_ex(model_dir.encode(), precision, devices.encode() if devices else None)
        if not self.h:
            raise RuntimeError("laya_create failed for %s" % model_dir)
        self.n_act = L.laya_n_act(self.h)
        self.max_markers = L.laya_max_markers(self.h)
        self.max_len = L.laya_max_len(self.h)
        self.num_devices = L.laya_num_devices(self.h)

    def close(self):
        if self.h:
            self.lib.laya_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward_batch(self, seqs: Sequence[Sequence[int]], markers: Sequence[Sequence[int]], qtypes: Sequence[int]):
        """All questions in one engine call. Returns per-question logits and the [B, n_act] act logits.
        Raises ValueError when the engine rejects the batch (the reference's -1 contract)."""
        lo, ac, rc = self.forward_batch_raw(seqs, markers, qtypes)
        if rc != 0:
            raise ValueError("engine rejected batch (sequence too long or too many options)" if rc == -1
                             else "engine error %d" % rc)
        out, off = [], 0
        for m in markers:
            out.append(lo[off:off + len(m)])
            off += len(m)
        return out, ac

    def forward_batch_raw(self, seqs, markers, qtypes):
        B = len(seqs)
        lens, lp = _ia([len(s) for s in seqs])
        nm, np_ = _ia([len(m) for m in markers])
        ids, ip = _ia(list(itertools.chain.from_iterable(seqs)) or [0])
        mk, mp = _ia(list(itertools.chain.from_iterable(markers)) or [0])
        qt, qp = _ia(qtypes)
        lo = np.zeros(max(1, int(nm.sum())), dtype=np.float32)
        ac = np.zeros((max(1, B), self.n_act), dtype=np.float32)
        rc = self.lib.laya_forward_batch(self.h, B, lp, ip, np_, mp, qp, lo.ctypes.data_as(_FP), ac.ctypes.data_as(_FP))
        return lo[:int(nm.sum())], ac[:B], rc

    def temperature(self, qtype: int) -> float:
        return float(self.lib.laya_temperature(self.h, qtype))

    def tune_all(self):
        self.lib.laya_tune_all(self.h)

    def set_dump_dir(self, path):
        return self.lib.laya_set_dump_dir(self.h, path.encode() if path else None)
