"""Build the memory-layer CUDA library in-tree (``model_b200/libmemlayer.so``).

Every ``csrc/*.cu`` file is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) and linked into one shared
library that exports the C ABI of ``include/memlayer.h``.  nvcc
cross-compiles without a GPU, so this runs on any machine with CUDA 12.9.
"""

from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libmemlayer.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", INCLUDE, "-I", CSRC]


def _stale(obj: str, deps) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    objs, jobs = [], []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if _stale(obj, [src, *headers]):
            cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
            if ptxas_verbose:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed ({' '.join(cmd)}):\n{r.stdout}\n{r.stderr}")
        return r.stdout + r.stderr

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        for out in ex.map(run, jobs):
            if verbose and out.strip():
                print(out)
    if jobs or not os.path.exists(LIB):
        run([NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcudart_static", "-Xlinker",
             "-rpath=/usr/local/cuda/lib64", "-lrt", "-ldl", "-lpthread"])
    # the XLA FFI handlers of the JAX binding, where JAX is installed
    from model_b200 import jax_ffi
    jax_ffi.build(verbose=verbose)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_verbose="-v" in sys.argv))
