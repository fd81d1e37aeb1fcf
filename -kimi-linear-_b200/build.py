"""Build ``libkda_b200.so`` (the C-ABI CUDA library) in-tree with nvcc.

    python -m <package>.build      or      build.build(verbose=True)

Every ``csrc/*.cu`` is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/`` next to this
file, then linked into ``libkda_b200.so`` beside it (static CUDA runtime, so
the library does not depend on which libcudart the host process loaded).  A
translation unit is rebuilt when it or any header under ``csrc/`` or
``include/`` is newer than its object file.
"""

from __future__ import annotations

import concurrent.futures
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libkda_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-I", os.path.join(REPO, "include"), "-I", CSRC]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put CUDA's bin directory on PATH")


def _headers():
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(REPO, "include", "*.h")))


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose and res.stdout:
        print(res.stdout, end="")
    if res.returncode != 0 or (verbose and res.stderr):
        sys.stderr.write(res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"command failed ({res.returncode}): {' '.join(cmd)}")
    return res


def build(verbose: bool = False, ptxas_verbose: bool = False, force: bool = False) -> str:
    """Compile and link; returns the path of ``libkda_b200.so``."""
    nvcc = nvcc_path()
    os.makedirs(BUILD, exist_ok=True)
    hdr_mtime = max([os.path.getmtime(h) for h in _headers()] + [0.0])
    objs = []
    relinked = force or not os.path.exists(LIB)
    jobs = []
    for src in sorted(glob.glob(os.path.join(CSRC, "*.cu"))):
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        stale = (force or not os.path.exists(obj)
                 or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr_mtime))
        if stale:
            cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)
    if jobs:
        # translation units compile independently: one nvcc per unit at once
        with concurrent.futures.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 1)) as ex:
            for f in [ex.submit(_run, cmd, verbose) for cmd in jobs]:
                f.result()
        relinked = True
    if relinked or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        _run([nvcc, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs], verbose)
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_verbose="-v" in sys.argv, force="--force" in sys.argv)
