"""Build libflagattn_b200.so in-tree with nvcc for sm_100a.

``python -m flagattention_b200.build`` (or ``build()``) compiles every
``csrc/*.cu`` to an object in parallel and links one shared library next to
this file.  Rebuilds only when a source, header or this script is newer than
the library.
"""

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJDIR = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libflagattn_b200.so")
# The abort-path test library: the same objects except the MLA decode, built
# with FA_DEBUG_ABORT_TEST (short wait limit, one lost barrier arrival).  Only
# tests/test_gpu_abort.py loads it, in a child process.
ABORT_TEST_LIB = os.path.join(PKG, "libflagattn_b200_aborttest.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", INCLUDE, "-I", CSRC]


def _nvcc():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return _sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h")) + [os.path.abspath(__file__)]


def up_to_date():
    for lib in (LIB, ABORT_TEST_LIB):
        if not os.path.exists(lib):
            return False
        t = os.path.getmtime(lib)
        if not all(os.path.getmtime(d) <= t for d in _deps()):
            return False
    return True


def _compile(src, verbose_ptxas, defines=(), suffix=""):
    obj = os.path.join(OBJDIR, os.path.basename(src) + suffix + ".o")
    cmd = [_nvcc(), *ARCH, *FLAGS, *[f"-D{d}" for d in defines], "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(force=False, verbose_ptxas=False):
    """Compile and link; returns the library path."""
    if not force and not verbose_ptxas and up_to_date():
        return LIB
    os.makedirs(OBJDIR, exist_ok=True)
    srcs = _sources()
    mla = os.path.join(CSRC, "mla_sv.cu")
    jobs = [(s, (), "") for s in srcs] + [(mla, ("FA_DEBUG_ABORT_TEST",), ".aborttest")]
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
        results = list(ex.map(lambda j: _compile(j[0], verbose_ptxas, j[1], j[2]), jobs))
    if verbose_ptxas:
        for _, log in results[:len(srcs)]:
            sys.stderr.write(log)
    objs = [o for o, _ in results[:len(srcs)]]
    test_objs = [results[-1][0] if o.endswith("mla_sv.cu.o") else o for o in objs]
    for lib, parts in ((LIB, objs), (ABORT_TEST_LIB, test_objs)):
        tmp = lib + ".tmp"
        cmd = [_nvcc(), *ARCH, "-shared", "-o", tmp, *parts, "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, lib)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="--ptxas" in sys.argv))
