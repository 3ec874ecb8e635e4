"""Builds the sm_100a CUDA library ``libmsx_b200.so`` in-tree.

Usage: ``python mlx-sparse_b200/build.py [--force]``. Every ``csrc/*.cu`` file is
compiled with nvcc for ``sm_100a`` (objects under ``_build/``, rebuilt only when
a source or header is newer) and linked into
``mlx-sparse_b200/mlx_sparse/_lib/libmsx_b200.so`` next to the Python package,
so the library travels with the repository instead of living in a JIT cache.
"""

from __future__ import annotations

import concurrent.futures
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "mlx_sparse", "_lib")
LIB = os.path.join(LIB_DIR, "libmsx_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nccl_dirs():
    try:
        import nvidia.nccl  # type: ignore

        base = list(nvidia.nccl.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except Exception:
        pass
    return None, None


def _nvcc():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def _flags():
    flags = ARCH + [
        "-O3",
        "-lineinfo",
        "-std=c++17",
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        # host-side float arithmetic that restates the reference (solver
        # coefficients) keeps one rounding per operation
        "-Xcompiler",
        "-ffp-contract=off",
        "--expt-relaxed-constexpr",
        "-DMSX_SM=100",
        "-I" + INCLUDE,
        "-I" + CSRC,
    ]
    inc, _ = _nccl_dirs()
    if inc:
        flags += ["-I" + inc, "-DMSX_HAVE_NCCL=1"]
    return flags


def _newest_header():
    heads = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    return max((os.path.getmtime(h) for h in heads), default=0.0)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    nvcc = _nvcc()
    flags = _flags()
    head_time = _newest_header()
    objs = []
    jobs = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        stale = force or not os.path.exists(obj)
        if not stale:
            t = os.path.getmtime(obj)
            stale = t < os.path.getmtime(src) or t < head_time
        if stale:
            jobs.append([nvcc, "-c", src, "-o", obj] + flags)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {cmd[2]}:\n{r.stdout}\n{r.stderr}")
        return r.stderr

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for err in ex.map(run, jobs):
            if verbose and err:
                print(err, flush=True)

    lib_stale = force or bool(jobs) or not os.path.exists(LIB)
    if not lib_stale:
        lt = os.path.getmtime(LIB)
        lib_stale = any(os.path.getmtime(o) > lt for o in objs)
    if lib_stale:
        link = [nvcc, "-shared", "-o", LIB] + objs + ARCH + ["-lcudart"]
        _, nccl_lib = _nccl_dirs()
        if nccl_lib:
            link += ["-L" + nccl_lib, "-l:libnccl.so.2", "-Xlinker", "-rpath=" + nccl_lib]
        run(link)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
