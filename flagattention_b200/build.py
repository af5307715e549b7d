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
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(d) <= t for d in _deps())


def _compile(src, verbose_ptxas):
    obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
    cmd = [_nvcc(), *ARCH, *FLAGS, "-c", src, "-o", obj]
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
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    if verbose_ptxas:
        for _, log in results:
            sys.stderr.write(log)
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), *ARCH, "-shared", "-o", tmp, *[o for o, _ in results], "-lcuda"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="--ptxas" in sys.argv))
