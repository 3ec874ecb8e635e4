"""Generates ``pcg_poisson3d.json``: the CPU oracle's Jacobi-PCG result on the
BASELINE CG configuration (3D 7-point Poisson, 256^3 grid, b = A x* with
x* ~ U(-1, 1) from seed 1, x0 = 0, inv_diag = 1/6, rtol 1e-6, atol 0,
maxiter 2000) and on a 64^3 grid with the same recipe. The oracle restates the
reference's serial loop (src/preconditioners/pcg/pcg.cpp:70-230), so its
status and iteration count are the reference's; the GPU solve must match the
status and come within +-2 iterations. The 256^3 solve takes a few minutes on
one core, hence a committed fixture.

    python tests/golden/make_pcg_golden.py
"""

import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:0] = [os.path.dirname(HERE), os.path.dirname(os.path.dirname(HERE))]

import workloads as wl  # noqa: E402
from oracle import oracle  # noqa: E402


def solve(m):
    (d, i, p), (n, _) = wl.poisson3d(m)
    xs = wl.uniform_vector(n, 1)
    b = oracle.csr_matvec(d, i, p, xs, n)
    inv = np.full(n, 1.0 / 6.0, np.float32)
    t0 = time.time()
    x, info, res, its = oracle.csr_pcg_jacobi(d, i, p, b, np.zeros(n, np.float32), inv, rtol=1e-6, atol=0.0,
                                              maxiter=2000)
    return {"grid": m, "n": n, "nnz": int(d.size), "info": info, "residual": res, "iterations": its,
            "b_norm": float(np.linalg.norm(b.astype(np.float64))), "seconds_1core": round(time.time() - t0, 1),
            "x_head": x[:8].tolist()}


if __name__ == "__main__":
    out = {str(m): solve(m) for m in (64, 256)}
    with open(os.path.join(HERE, "pcg_poisson3d.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(json.dumps(out))
