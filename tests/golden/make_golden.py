"""Generates ``reference_cases.json``: the known-answer cases of mlx-sparse's own
tests for the product path, with their expected outputs.

Each case restates one reference test's inputs (cited by file:line in that
project's ``tests/`` tree) and records the expected result the test asserts:
hand-computed values where the test states them, otherwise the SciPy result
the test compares against (SciPy is the reference tests' secondary oracle).
Run once with SciPy available; the JSON is committed so the GPU box needs
neither SciPy nor the reference tree.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import json
import os

import numpy as np
import scipy.sparse as sp
import scipy.sparse.linalg as spla

HERE = os.path.dirname(os.path.abspath(__file__))


def _csr(m):
    m = m.tocsr()
    m.sort_indices()
    return {"data": m.data.astype(np.float32).tolist(), "indices": m.indices.astype(np.int64).tolist(),
            "indptr": m.indptr.astype(np.int64).tolist(), "shape": list(m.shape)}


def main():
    cases = {}

    # tests/test_csr_matvec.py:25-36
    cases["spmv_hand"] = {
        "A": {"data": [2.0, -1.0, 4.0, 5.0], "indices": [0, 2, 1, 3], "indptr": [0, 2, 2, 4], "shape": [3, 4]},
        "x": [3.0, 10.0, 7.0, -2.0],
        "y": [-1.0, 0.0, 30.0],
        "source": "tests/test_csr_matvec.py:25-36",
    }
    # tests/test_csr_matvec.py:39-63
    rng = np.random.default_rng(456)
    A = sp.random(96, 128, density=0.03, format="csr", dtype=np.float32, random_state=rng)
    x = rng.normal(size=(128,)).astype(np.float32)
    cases["spmv_scipy_456"] = {"A": _csr(A), "x": x.tolist(), "y": (A @ x).astype(np.float32).tolist(),
                               "source": "tests/test_csr_matvec.py:39-63"}

    # tests/test_csr_matmul.py:25-45
    cases["spmm_hand"] = {
        "A": {"data": [2.0, -1.0, 4.0, 5.0], "indices": [0, 2, 1, 3], "indptr": [0, 2, 2, 4], "shape": [3, 4]},
        "B": [[3.0, 1.0], [10.0, -2.0], [7.0, 4.0], [-2.0, 6.0]],
        "Y": [[-1.0, -2.0], [0.0, 0.0], [30.0, 22.0]],
        "source": "tests/test_csr_matmul.py:25-45",
    }
    # tests/test_csr_matmul.py:48-76
    rng = np.random.default_rng(789)
    A = sp.random(64, 80, density=0.04, format="csr", dtype=np.float32, random_state=rng)
    B = rng.normal(size=(80, 7)).astype(np.float32)
    cases["spmm_scipy_789"] = {"A": _csr(A), "B": B.tolist(), "Y": (A @ B).astype(np.float32).tolist(),
                               "source": "tests/test_csr_matmul.py:48-76"}
    # tests/test_csr_matmul.py:156-217 (fp16 5e-3 / bf16 3e-2 tolerances)
    data = np.array([0.5, -2.0, 3.0, 1.25, -0.75, 4.0], dtype=np.float32)
    A = sp.csr_matrix((data, np.array([0, 3, 1, 4, 2, 3]), np.array([0, 2, 4, 6])), shape=(3, 5))
    B = np.array([[1.0, -0.5, 2.0, 0.25], [-1.5, 0.75, 1.25, 2.5], [0.5, -2.0, 3.0, -0.75],
                  [2.0, 1.5, -1.0, 0.5], [-0.25, 1.0, 0.75, -1.25]], dtype=np.float32)
    cases["spmm_lowp"] = {"A": _csr(A), "B": B.tolist(), "Y": (A @ B).astype(np.float32).tolist(),
                          "tol": {"float16": 5e-3, "bfloat16": 3e-2},
                          "source": "tests/test_csr_matmul.py:156-217"}

    # tests/test_csr_matmul.py:383-432 (exact cancellation is pruned)
    lhs = sp.csr_matrix((np.array([1.0, -1.0, 2.0, 3.0, -2.0], np.float32), np.array([1, 2, 0, 2, 3]),
                         np.array([0, 2, 3, 5])), shape=(3, 4))
    rhs = sp.csr_matrix((np.array([4.0, 7.0, -7.0, 5.0, -3.0, 3.0], np.float32), np.array([2, 0, 0, 1, 2, 2]),
                         np.array([0, 1, 3, 4, 6])), shape=(4, 3))
    C = (lhs @ rhs).tocsr()
    C.eliminate_zeros()
    cases["spgemm_cancel"] = {"A": _csr(lhs), "B": _csr(rhs), "C": _csr(C),
                              "source": "tests/test_csr_matmul.py:383-432"}
    # tests/test_csr_matmul.py:480-517 (reversed blocks -> sorted columns)
    block, blocks = 8, 16
    lhs = sp.csr_matrix((np.ones(blocks, np.float32), np.arange(blocks), np.array([0, blocks])), shape=(1, blocks))
    ri = np.concatenate([np.arange((blocks - r - 1) * block, (blocks - r) * block) for r in range(blocks)])
    rd = np.linspace(0.5, 2.0, ri.size, dtype=np.float32)
    rhs = sp.csr_matrix((rd, ri, np.arange(blocks + 1) * block), shape=(blocks, block * blocks))
    rhs_raw = {"data": rd.tolist(), "indices": ri.tolist(), "indptr": (np.arange(blocks + 1) * block).tolist(),
               "shape": [blocks, block * blocks]}
    C = (lhs @ rhs).tocsr()
    cases["spgemm_dense_ordered"] = {"A": _csr(lhs), "B": rhs_raw, "C": _csr(C),
                                     "source": "tests/test_csr_matmul.py:480-517"}

    # tests/test_linalg_preconditioners.py:257-266,1977-1987
    cases["pcg_2x2"] = {
        "A": {"data": [4.0, 1.0, 1.0, 3.0], "indices": [0, 1, 0, 1], "indptr": [0, 2, 4], "shape": [2, 2]},
        "b": [1.0, 2.0], "x": [1.0 / 11.0, 7.0 / 11.0], "rtol": 1e-6, "atol": 0.0, "maxiter": 32,
        "source": "tests/test_linalg_preconditioners.py:1977-1987",
    }
    # tests/test_linalg_preconditioners.py:1990-2019
    A_dense = np.array([[6.0, 1.0, 0.0, 0.0], [1.0, 5.0, 1.0, 0.0], [0.0, 1.0, 4.0, 1.0], [0.0, 0.0, 1.0, 3.0]],
                       dtype=np.float32)
    b = np.array([1.0, 2.0, -1.0, 0.5], dtype=np.float32)
    cases["pcg_4x4"] = {"A": _csr(sp.csr_matrix(A_dense)), "b": b.tolist(),
                        "x": np.linalg.solve(A_dense.astype(np.float64), b.astype(np.float64)).tolist(),
                        "rtol": 1e-7, "atol": 1e-8, "maxiter": 32,
                        "source": "tests/test_linalg_preconditioners.py:1990-2019"}
    # tests/test_linalg_preconditioners.py:2022-2070
    n = 8
    poisson = sp.diags([-np.ones(n - 1), 2.5 * np.ones(n), -np.ones(n - 1)], offsets=[-1, 0, 1], format="csr",
                       dtype=np.float32)
    scaling = np.geomspace(1.0e-1, 1.0e1, n).astype(np.float32)
    D = sp.diags(scaling, format="csr", dtype=np.float32)
    sA = (D @ poisson @ D).astype(np.float32).tocsr()
    x_true = np.linspace(-1.0, 1.0, n, dtype=np.float32)
    b = (sA @ x_true).astype(np.float32)
    inv_diag = 1.0 / sA.diagonal()
    M = spla.LinearOperator(sA.shape, matvec=lambda v: inv_diag * v, dtype=np.float32)
    x_sp, info = spla.cg(sA, b, M=M, rtol=1e-5, atol=1e-7, maxiter=64)
    assert info == 0
    cases["pcg_scaled_poisson"] = {"A": _csr(sA), "b": b.tolist(), "x": x_sp.astype(np.float32).tolist(),
                                   "rtol": 1e-5, "atol": 1e-7, "maxiter": 64, "x_tol": 2e-3,
                                   "source": "tests/test_linalg_preconditioners.py:2022-2070"}
    # tests/test_linalg_preconditioners.py:269-278,2094-2123
    cases["pcg_diag"] = {
        "A": {"data": [1.0e-6, 1.0, 10.0], "indices": [0, 1, 2], "indptr": [0, 1, 2, 3], "shape": [3, 3]},
        "b": [1.0, 2.0, 30.0], "x": [1.0e6, 2.0, 3.0], "rtol": 1e-6, "atol": 1e-8, "maxiter": 16,
        "max_iterations": 2,
        "source": "tests/test_linalg_preconditioners.py:2094-2123",
    }

    # tests/test_coo_tocsr.py:23-36 (sorted by row, then column)
    cases["coo_tocsr_sort"] = {
        "data": [10.0, 20.0, 30.0, 40.0], "row": [2, 0, 1, 0], "col": [1, 3, 2, 0], "shape": [3, 4],
        "indptr": [0, 2, 3, 4], "indices": [0, 3, 2, 1], "out_data": [40.0, 20.0, 30.0, 10.0],
        "source": "tests/test_coo_tocsr.py:23-36",
    }
    # tests/test_coo_tocsr.py:38-51 (duplicates summed by canonicalize)
    cases["coo_canonical_dups"] = {
        "data": [2.0, 3.0, 5.0], "row": [0, 0, 0], "col": [1, 1, 0], "shape": [1, 3],
        "indptr": [0, 2], "indices": [0, 1], "out_data": [5.0, 5.0],
        "source": "tests/test_coo_tocsr.py:38-51",
    }
    # tests/test_coo_tocsr.py:53-60 (empty)
    cases["coo_empty"] = {"data": [], "row": [], "col": [], "shape": [4, 5], "indptr": [0, 0, 0, 0, 0],
                          "indices": [], "out_data": [], "source": "tests/test_coo_tocsr.py:53-60"}

    # tests/test_grad.py:180-223 (loss = sum((A x)^2); gradients of the dense
    # product restricted to the stored coordinates, as the test compares)
    row = np.array([0, 0, 2, 2])
    col = np.array([0, 2, 1, 3])
    vals = np.array([2.0, -1.0, 4.0, 5.0])
    dense = np.zeros((3, 4))
    dense[row, col] = vals
    x = np.array([3.0, 10.0, 7.0, -2.0])
    y = dense @ x
    cases["grad_csr_matvec"] = {
        "A": {"data": vals.tolist(), "indices": col.tolist(), "indptr": [0, 2, 2, 4], "shape": [3, 4]},
        "x": x.tolist(), "grad_data": (2 * y[row] * x[col]).tolist(), "grad_x": (2 * dense.T @ y).tolist(),
        "source": "tests/test_grad.py:180-223",
    }
    # tests/test_grad.py:358-404 (COO @ B, loss = sum(Y^2))
    row = np.array([0, 0, 1, 2, 2])
    col = np.array([0, 2, 1, 0, 3])
    vals = np.array([2.0, -1.0, 0.5, 3.0, -2.0])
    B = np.arange(12, dtype=np.float64).reshape(4, 3) / 7.0
    dense = np.zeros((3, 4))
    dense[row, col] = vals
    Y = dense @ B
    cases["grad_coo_matmul"] = {
        "data": vals.tolist(), "row": row.tolist(), "col": col.tolist(), "shape": [3, 4],
        "B": B.astype(np.float32).tolist(), "grad_data": (2 * np.sum(Y[row] * B[col], axis=1)).tolist(),
        "grad_B": (2 * dense.T @ Y).tolist(), "source": "tests/test_grad.py:358-404",
    }

    path = os.path.join(HERE, "reference_cases.json")
    with open(path, "w") as f:
        json.dump(cases, f, indent=1)
    print(path)


if __name__ == "__main__":
    main()
