"""Builds the engine shared library ``layamd_b200/liblaya_b200.so`` from ``layamd_b200/csrc``.

Every translation unit is compiled by nvcc for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``); the library links the CUDA runtime statically, so it only needs
the driver at run time. Objects go to ``layamd_b200/_build`` and are rebuilt when a source or header
is newer than them. Usage: ``python -m layamd_b200.build [-j N] [--force] [--debug-bounds]``;
``--debug-bounds`` builds ``liblaya_b200_dbg.so`` (objects in ``_build_dbg``) with -DLAYA_DEBUG_BOUNDS,
whose kernels check every index they read from the packing maps.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "liblaya_b200.so")
# debug bounds build: every kernel checks the indices it reads from the packing maps
BUILD_DBG = os.path.join(HERE, "_build_dbg")
LIB_DBG = os.path.join(HERE, "liblaya_b200_dbg.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3,-Wall",
              "--expt-relaxed-constexpr", "-I" + CSRC, "-I" + os.path.join(os.path.dirname(HERE), "include")]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def _headers():
    return glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(CSRC, "*.hpp")) + glob.glob(os.path.join(os.path.dirname(HERE), "include", "*.h"))


def _stale(obj, src, hdr_mtime):
    return not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr_mtime)


def build(jobs=None, force=False, verbose=False, debug_bounds=False):
    """Compile stale objects and relink the library when anything changed. Returns the .so path.
    debug_bounds: the debug bounds build (-DLAYA_DEBUG_BOUNDS) into liblaya_b200_dbg.so instead."""
    bdir, lib = (BUILD_DBG, LIB_DBG) if debug_bounds else (BUILD, LIB)
    flags = NVCC_FLAGS + (["-DLAYA_DEBUG_BOUNDS"] if debug_bounds else [])
    os.makedirs(bdir, exist_ok=True)
    nvcc = _nvcc()
    hdr_mtime = max([os.path.getmtime(h) for h in _headers()] + [0])
    srcs = _sources()
    objs = [os.path.join(bdir, os.path.basename(s) + ".o") for s in srcs]
    todo = [(s, o) for s, o in zip(srcs, objs) if force or _stale(o, s, hdr_mtime)]

    def cc(pair):
        src, obj = pair
        cmd = [nvcc] + ARCH + flags + ["-c", src, "-o", obj]
        if src.endswith(".cpp"):
            cmd[1:1] = ["-x", "cu"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed for %s:\n%s%s" % (src, r.stdout, r.stderr))
        if verbose and (r.stdout or r.stderr):
            sys.stderr.write(r.stdout + r.stderr)
        return obj

    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
            list(ex.map(cc, todo))
    if todo or not os.path.exists(lib) or any(os.path.getmtime(o) > os.path.getmtime(lib) for o in objs):
        tmp = lib + ".tmp"
        cmd = [nvcc] + ARCH + ["-shared", "-Xcompiler", "-fPIC", "-o", tmp] + objs + ["-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s%s" % (r.stdout, r.stderr))
        os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", action="store_true")
    ap.add_argument("--debug-bounds", action="store_true", help="build liblaya_b200_dbg.so (device index checks)")
    a = ap.parse_args()
    print(build(a.j, a.force, a.v, a.debug_bounds))
