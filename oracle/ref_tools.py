"""Builds the reference's own C++ host tools, unmodified, against this library.

Test infrastructure, not product: the reference ships two programs that link its engine library
through ``src/laya_api.h`` -- the benchmark ``src/bench_engine.cpp`` (per-call p50 of single questions
and of batches) and the golden-set checker ``src/test_parity.cpp``. Each is compiled here from its own
source file where it lies in the reference checkout (``LAYA_REFERENCE``), in a wrapper translation
unit that includes this repository's ``include/laya_api.h`` first: the reference's header is then
included as well, so any declaration whose signature differs between the two is a compile error.
The program is linked against ``layamd_b200/liblaya_b200.so`` (found through an rpath relative to
the binary) and written to ``oracle/_ref/`` (git-ignored; it travels with the repository to a GPU
box, where the reference checkout does not exist). Nothing of the reference is copied into this
repository.

Usage: ``python -m oracle.ref_tools`` (also run by ``__graft_entry__.build()`` when the reference
checkout is present).
"""
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OUT = os.path.join(ROOT, "oracle", "_ref")
TOOLS = ("bench_engine", "test_parity")


def reference_root():
    """The reference checkout: LAYA_REFERENCE, else a directory named ``reference`` beside this
    repository's root."""
    return os.environ.get("LAYA_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference")


def reference_src():
    return os.path.join(reference_root(), "src")


def wrapper_source(tool, ref_src=None):
    """The translation unit that compiles reference tool `tool` against this repository's header."""
    ref_src = ref_src or reference_src()
    return '#include "%s"\n#include "%s"\n' % (os.path.join(ROOT, "include", "laya_api.h"),
                                               os.path.join(ref_src, tool + ".cpp"))


def build_tool(tool, out_dir=OUT, ref_src=None, link=True):
    """Compiles (and links, unless link=False) one reference tool; returns the output path. Raises
    CalledProcessError with the compiler's message on failure."""
    os.makedirs(out_dir, exist_ok=True)
    w = os.path.join(out_dir, "w_%s.cpp" % tool)
    with open(w, "w") as f:
        f.write(wrapper_source(tool, ref_src))
    lib_dir = os.path.join(ROOT, "layamd_b200")
    if link:
        out = os.path.join(out_dir, tool)
        rpath = os.path.relpath(lib_dir, out_dir)
        cmd = ["g++", "-std=c++17", "-O2", w, "-o", out, "-L" + lib_dir, "-llaya_b200",
               "-Wl,-rpath,$ORIGIN/" + rpath]
    else:
        out = os.path.join(out_dir, tool + ".o")
        cmd = ["g++", "-std=c++17", "-O2", "-c", w, "-o", out]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return out


def build(out_dir=OUT):
    """Builds every tool when the reference checkout is present; returns the built paths."""
    if not os.path.isdir(reference_src()):
        return []
    return [build_tool(t, out_dir) for t in TOOLS]


if __name__ == "__main__":
    for p in build():
        print(p)
    sys.exit(0)
