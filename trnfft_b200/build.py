"""Build the trnfft_b200 CUDA library in-tree.

``python -m trnfft_b200.build`` (or ``build()``) compiles every ``csrc/*.cu``
for sm_100a with nvcc and links ``trnfft_b200/_lib/libtrnfft_b200.so``, the
C-ABI library declared in ``include/trnfft_b200.h``.  Rebuilds only what is
older than its sources.
"""

from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT_DIR = os.path.join(HERE, "_lib")
OBJ_DIR = os.path.join(OUT_DIR, "obj")
LIB = os.path.join(OUT_DIR, "libtrnfft_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-rdc=true", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I" + os.path.join(ROOT, "include"),
] + ARCH


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the trnfft_b200 CUDA library cannot be built")


def _deps(src: str) -> list[str]:
    hdrs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    hdrs += glob.glob(os.path.join(ROOT, "include", "*.h"))
    return [src] + hdrs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_verbose: bool = False) -> str:
    """Compile and link the library; returns its path."""
    nvcc = _nvcc()
    os.makedirs(OBJ_DIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    jobs = []
    for s in srcs:
        obj = os.path.join(OBJ_DIR, os.path.basename(s)[:-3] + ".o")
        if _stale(obj, _deps(s)):
            cmd = [nvcc, *NVCC_FLAGS, "-c", s, "-o", obj]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append((s, cmd))

    def run(job):
        s, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        return s, r

    failed = []
    with ThreadPoolExecutor(max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        for s, r in ex.map(run, jobs):
            if r.returncode != 0:
                failed.append((s, r.stderr))
            elif verbose or ptxas_verbose:
                sys.stderr.write(r.stderr)
    if failed:
        msg = "\n".join(f"--- {s}\n{err}" for s, err in failed)
        raise RuntimeError("nvcc failed:\n" + msg)
    objs = [os.path.join(OBJ_DIR, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if _stale(LIB, objs):
        cmd = [nvcc, "-shared", "-rdc=true", *ARCH, *objs, "-o", LIB, "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv))
