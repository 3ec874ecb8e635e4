"""Pins the CPU oracle: reference known answers, SciPy, determinism.

CPU only. The oracle is trusted as the GPU parity checker only because it
reproduces every known-answer case of the reference's tests for this path
(tests/golden/reference_cases.json) and agrees with SciPy on seeded inputs.
"""

import os

import numpy as np
import pytest
import scipy.sparse as sp

import workloads as wl


def _arr(A, it=np.int32):
    return (np.asarray(A["data"], np.float32), np.asarray(A["indices"], it), np.asarray(A["indptr"], it))


@pytest.mark.parametrize("it", [np.int32, np.int64])
def test_spmv_known_answers(orc, golden, it):
    for name in ("spmv_hand", "spmv_scipy_456"):
        c = golden[name]
        d, i, p = _arr(c["A"], it)
        y = orc.csr_matvec(d, i, p, np.asarray(c["x"], np.float32), c["A"]["shape"][0])
        np.testing.assert_allclose(y, np.asarray(c["y"], np.float32), rtol=1e-5, atol=1e-5)


def test_spmm_known_answers(orc, golden):
    for name in ("spmm_hand", "spmm_scipy_789", "spmm_lowp"):
        c = golden[name]
        d, i, p = _arr(c["A"])
        Y = orc.csr_matmul(d, i, p, np.asarray(c["B"], np.float32), c["A"]["shape"][0])
        np.testing.assert_allclose(Y, np.asarray(c["Y"], np.float32), rtol=1e-5, atol=1e-5)


def test_spmm_low_precision(orc, golden):
    c = golden["spmm_lowp"]
    d, i, p = _arr(c["A"])
    B = np.asarray(c["B"], np.float32)
    Y16 = orc.csr_matmul(d.astype(np.float16), i, p, B.astype(np.float16), 3)
    np.testing.assert_allclose(Y16.astype(np.float32), c["Y"], rtol=5e-3, atol=5e-3)
    Yb = orc.csr_matmul(orc.f32_to_bf16_bits(d), i, p, orc.f32_to_bf16_bits(B), 3, bf16=True)
    np.testing.assert_allclose(orc.bf16_bits_to_f32(Yb), c["Y"], rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("name", ["spgemm_cancel", "spgemm_dense_ordered"])
def test_spgemm_known_answers(orc, golden, name):
    c = golden[name]
    a, b = _arr(c["A"]), _arr(c["B"])
    d, i, p = orc.csr_matmat(a, b, c["A"]["shape"], c["B"]["shape"])
    np.testing.assert_array_equal(i, c["C"]["indices"])
    np.testing.assert_array_equal(p, c["C"]["indptr"])
    np.testing.assert_allclose(d, c["C"]["data"], rtol=1e-5, atol=1e-5)
    assert np.all(d != 0)
    assert i.dtype == np.int32


def test_spgemm_mixed_index_dtype_gives_int64(orc, golden):
    c = golden["spgemm_cancel"]
    d, i, p = orc.csr_matmat(_arr(c["A"], np.int32), _arr(c["B"], np.int64), c["A"]["shape"], c["B"]["shape"])
    assert i.dtype == np.int64 and p.dtype == np.int64


def test_spgemm_matches_scipy_random(orc):
    (ad, ai, ap), sa = wl.random_csr(50, 60, 0.08, seed=11)
    (bd, bi, bp), sb = wl.random_csr(60, 70, 0.08, seed=12)
    d, i, p = orc.csr_matmat((ad, ai, ap), (bd, bi, bp), sa, sb)
    C = (sp.csr_matrix((ad, ai, ap), shape=sa) @ sp.csr_matrix((bd, bi, bp), shape=sb)).tocsr()
    C.eliminate_zeros()
    C.sort_indices()
    np.testing.assert_array_equal(i, C.indices)
    np.testing.assert_array_equal(p, C.indptr)
    np.testing.assert_allclose(d, C.data, rtol=1e-5, atol=1e-6)


def test_pcg_known_answers(orc, golden):
    for name in ("pcg_2x2", "pcg_4x4", "pcg_scaled_poisson", "pcg_diag"):
        c = golden[name]
        d, i, p = _arr(c["A"])
        n = c["A"]["shape"][0]
        A = sp.csr_matrix((d, i, p), shape=(n, n))
        inv = (1.0 / A.diagonal()).astype(np.float32)
        b = np.asarray(c["b"], np.float32)
        x, info, res, its = orc.csr_pcg_jacobi(d, i, p, b, np.zeros(n, np.float32), inv, rtol=c["rtol"],
                                               atol=c["atol"], maxiter=c["maxiter"])
        assert info == 0, name
        tol = c.get("x_tol", 1e-4)
        np.testing.assert_allclose(x, c["x"], rtol=tol, atol=tol)
        if "max_iterations" in c:
            assert its <= c["max_iterations"]
            assert res == pytest.approx(np.linalg.norm(A @ x - b), abs=1e-4)


def test_cg_matches_scipy(orc):
    (d, i, p), (n, _) = wl.lap2d(12)
    A = sp.csr_matrix((d, i, p), shape=(n, n))
    b = wl.uniform_vector(n, 5)
    x, info, res, its = orc.csr_cg(d, i, p, b, np.zeros(n, np.float32), rtol=1e-6, atol=0.0, maxiter=500)
    assert info == 0 and its > 0
    ref = np.linalg.solve(A.toarray().astype(np.float64), b.astype(np.float64))
    np.testing.assert_allclose(x, ref, rtol=1e-4, atol=1e-4)
    assert res == pytest.approx(np.linalg.norm(b - A @ x), rel=1e-2, abs=1e-5)


def test_cg_status_codes(orc):
    # maxiter exhausted -> info == maxiter; maxiter == 0 -> info == 1 (cg.cpp:150)
    (d, i, p), (n, _) = wl.lap2d(10)
    b = wl.uniform_vector(n, 1)
    x0 = np.zeros(n, np.float32)
    _, info, _, its = orc.csr_cg(d, i, p, b, x0, rtol=1e-12, atol=0.0, maxiter=3)
    assert info == 3 and its == 3
    _, info, _, its = orc.csr_cg(d, i, p, b, x0, rtol=1e-12, atol=0.0, maxiter=0)
    assert info == 1 and its == 0
    # non-finite b -> -3
    bad = b.copy()
    bad[3] = np.inf
    _, info, _, _ = orc.csr_cg(d, i, p, bad, x0, rtol=1e-6, atol=0.0, maxiter=10)
    assert info == -3
    # indefinite preconditioner -> -2 (pcg.cpp:155-160)
    inv = np.full(n, -0.25, np.float32)
    _, info, _, _ = orc.csr_pcg_jacobi(d, i, p, b, x0, inv, rtol=1e-6, atol=0.0, maxiter=10)
    assert info == -2


@pytest.mark.parametrize("workers", [2, 3, 8])
def test_parallel_equals_serial(orc, workers):
    (d, i, p), (n, m) = wl.ragged_csr(3000, 400, seed=3, max_len=30, index_dtype=np.int64)
    x = wl.uniform_vector(m, 4)
    np.testing.assert_array_equal(orc.csr_matvec(d, i, p, x, n, workers=1),
                                  orc.csr_matvec(d, i, p, x, n, workers=workers))
    B = wl.uniform_matrix(m, 16, 6)
    np.testing.assert_array_equal(orc.csr_matmul(d, i, p, B, n, workers=1),
                                  orc.csr_matmul(d, i, p, B, n, workers=workers))


def test_weighted_ranges_balance(orc):
    work = np.array([1, 1, 1, 100, 1, 1, 1, 1], dtype=np.int64)
    r = orc.weighted_ranges(work, 3)
    assert r[0][0] == 0 and r[-1][1] == work.size
    assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
    assert len(orc.weighted_ranges(work, 1)) == 1


def test_workload_generators_are_canonical():
    for (d, i, p), shape in (wl.lap2d(16), wl.poisson3d(6), wl.random_k_per_row(100, 1000, 8, 2),
                             wl.power_law(500, 3), wl.ragged_csr(200, 100, 1, 10)):
        assert p[0] == 0 and p[-1] == d.size == i.size
        assert np.all(np.diff(p) >= 0)
        for r in range(shape[0]):
            row = i[p[r]:p[r + 1]]
            assert np.all(np.diff(row) > 0)
            assert row.size == 0 or (row[0] >= 0 and row[-1] < shape[1])


# The reference's SuiteSparse fixtures, read in place: MSX_REFERENCE_ROOT
# names the mlx-sparse checkout (default: a `reference` folder beside this
# repository).
_HB = os.path.join(os.environ.get("MSX_REFERENCE_ROOT", os.path.join(os.path.dirname(os.path.dirname(
    os.path.dirname(os.path.abspath(__file__)))), "reference")), "tests", "fixtures", "suitesparse", "HB")


def _hb_matrices():
    """Names of the reference's SuiteSparse fixtures; looked up only when a
    test that uses them runs (never at collection)."""
    import os

    if not os.path.isdir(_HB):
        pytest.skip("reference SuiteSparse fixtures not present")
    return sorted(f for f in os.listdir(_HB) if f.endswith(".mtx") and not f.endswith("_b.mtx"))


def test_oracle_on_reference_suitesparse_fixtures(orc):
    """The SuiteSparse Harwell-Boeing matrices the reference's tests ship
    (read in place, not copied): oracle SpMV / SpMM / SpGEMM against SciPy,
    the secondary oracle the reference's own tests use."""
    import os

    import scipy.io

    names = _hb_matrices()
    assert names
    for name in names:
        A = sp.csr_matrix(scipy.io.mmread(os.path.join(_HB, name))).astype(np.float32)
        A.sum_duplicates()
        A.sort_indices()
        d, i, p = A.data, A.indices.astype(np.int32), A.indptr.astype(np.int32)
        m, n = A.shape
        x = wl.uniform_vector(n, 3)
        y = orc.csr_matvec(d, i, p, x, m)
        scale = np.abs(A) @ np.abs(x) + 1e-30
        assert np.max(np.abs(y - A @ x) / np.maximum(np.abs(A @ x), scale)) <= 1e-5, name
        B = wl.uniform_matrix(n, 8, 4)
        np.testing.assert_allclose(orc.csr_matmul(d, i, p, B, m), A @ B, rtol=1e-4,
                                   atol=1e-4 * float(np.abs(A).max()), err_msg=name)
        if m == n:
            cd, ci, cp = orc.csr_matmat((d, i, p), (d, i, p), (m, n), (m, n))
            C = (A @ A).tocsr()
            C.eliminate_zeros()
            C.sort_indices()
            np.testing.assert_array_equal(ci, C.indices, err_msg=name)
            np.testing.assert_array_equal(cp, C.indptr, err_msg=name)


def test_oracle_pcg_on_bcsstk03():
    """Jacobi PCG on the SPD structural matrix bcsstk03: converged solutions
    satisfy the reference's stopping rule against a float64 check."""
    import os

    import scipy.io

    from oracle import oracle as orc

    if "bcsstk03.mtx" not in _hb_matrices():
        pytest.skip("bcsstk03 not present")
    path = os.path.join(_HB, "bcsstk03.mtx")
    A = sp.csr_matrix(scipy.io.mmread(path)).astype(np.float32)
    A.sum_duplicates()
    A.sort_indices()
    n = A.shape[0]
    d, i, p = A.data, A.indices.astype(np.int32), A.indptr.astype(np.int32)
    b = (A @ wl.uniform_vector(n, 1)).astype(np.float32)
    inv = (1.0 / A.diagonal()).astype(np.float32)
    x, info, res, its = orc.csr_pcg_jacobi(d, i, p, b, np.zeros(n, np.float32), inv, rtol=1e-5, atol=0.0,
                                           maxiter=10 * n)
    assert info in (0, -1, 10 * n)
    if info == 0:
        r = b.astype(np.float64) - A.astype(np.float64) @ x.astype(np.float64)
        assert np.linalg.norm(r) <= 1e-3 * np.linalg.norm(b)


def test_pcg_poisson3d_fixture_reproduces(orc):
    """The committed PCG fixture (tests/golden/pcg_poisson3d.json, which the
    GPU tests read for the 256^3 BASELINE solve) is the oracle's result: the
    64^3 entry is recomputed here (0.5 s) and must match exactly."""
    import json

    with open(os.path.join(os.path.dirname(__file__), "golden", "pcg_poisson3d.json")) as f:
        g = json.load(f)["64"]
    (d, i, p), (n, _) = wl.poisson3d(64)
    b = orc.csr_matvec(d, i, p, wl.uniform_vector(n, 1), n)
    x, info, res, its = orc.csr_pcg_jacobi(d, i, p, b, np.zeros(n, np.float32), np.full(n, 1.0 / 6.0, np.float32),
                                           rtol=1e-6, atol=0.0, maxiter=2000)
    assert (info, its) == (g["info"], g["iterations"])
    assert res == pytest.approx(g["residual"], rel=1e-6)
    assert x[:8].tolist() == g["x_head"]


@pytest.mark.parametrize("name", ["coo_tocsr_sort", "coo_empty"])
def test_coo_tocsr_known_answers(orc, golden, name):
    c = golden[name]
    d, i, p, _ = orc.coo_tocsr(np.asarray(c["data"], np.float32), np.asarray(c["row"], np.int32),
                               np.asarray(c["col"], np.int32), c["shape"][0])
    assert p.tolist() == c["indptr"] and i.tolist() == c["indices"] and d.tolist() == c["out_data"]


@pytest.mark.parametrize("it", [np.int32, np.int64])
def test_coo_oracle_matches_numpy_and_scipy(orc, it):
    rng = np.random.default_rng(3)
    n, m, nnz = 400, 300, 5000
    row = rng.integers(0, n, nnz).astype(it)
    col = rng.integers(0, m, nnz).astype(it)
    d = rng.standard_normal(nnz).astype(np.float32)
    od, oi, op, perm = orc.coo_tocsr(d, row, col, n)
    assert np.array_equal(perm, np.lexsort((np.arange(nnz), col, row)))  # (row, col, source) order
    assert np.array_equal(oi, col[perm]) and np.array_equal(od, d[perm])
    assert np.array_equal(op, np.concatenate([[0], np.cumsum(np.bincount(row, minlength=n))]))
    _, _, _, perm_s = orc.coo_tocsr(d, row, col, n, sort_columns=False)
    assert np.array_equal(perm_s, np.argsort(row, kind="stable"))
    S = sp.coo_matrix((d, (row, col)), shape=(n, m)).tocsr()
    x = wl.uniform_vector(m, 1)
    B = wl.uniform_matrix(m, 5, 2)
    np.testing.assert_allclose(orc.coo_matmul(d, row, col, x, n), S @ x, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(orc.coo_matmul(d, row, col, B, n), S @ B, rtol=1e-5, atol=1e-5)


def test_transpose_and_data_vjp_oracle_match_scipy(orc):
    (d, i, p), shape = wl.ragged_csr(300, 200, 4, 20)
    S = sp.csr_matrix((d, i, p), shape=shape)
    x = wl.uniform_vector(shape[0], 1)
    B = wl.uniform_matrix(shape[0], 4, 2)
    np.testing.assert_allclose(orc.csr_matmul_transpose(d, i, p, x, shape[1]), S.T @ x, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(orc.csr_matmul_transpose(d, i, p, B, shape[1]), S.T @ B, rtol=1e-5, atol=1e-5)
    xc, cot = wl.uniform_vector(shape[1], 3), wl.uniform_vector(shape[0], 4)
    rows = np.repeat(np.arange(shape[0]), np.diff(p))
    np.testing.assert_array_equal(orc.csr_data_vjp(i, p, xc, cot), cot[rows] * xc[i])
    Bc, C = wl.uniform_matrix(shape[1], 3, 5), wl.uniform_matrix(shape[0], 3, 6)
    np.testing.assert_allclose(orc.csr_data_vjp(i, p, Bc, C), np.sum(C[rows] * Bc[i], axis=1), rtol=1e-6, atol=1e-6)


def test_chebyshev_oracle_approaches_the_solve(orc):
    """A high-degree Chebyshev semi-iteration over the exact spectral
    interval approximates A^-1 r, and the oracle's Chebyshev PCG converges to
    SciPy's solution."""
    (d, i, p), shape = wl.lap2d(12)
    S = sp.csr_matrix((d, i, p), shape=shape).toarray().astype(np.float64)
    ev = np.linalg.eigvalsh(S)
    r = wl.uniform_vector(shape[0], 1)
    z = orc.chebyshev_apply(d, i, p, r, degree=60, lambda_min=float(ev[0]), lambda_max=float(ev[-1]))
    np.testing.assert_allclose(z, np.linalg.solve(S, r), rtol=1e-3, atol=1e-3)
    x, info, _, its = orc.csr_pcg_chebyshev(d, i, p, r, np.zeros(shape[0], np.float32), (d, i, p), degree=3,
                                            lambda_min=float(ev[0]), lambda_max=float(ev[-1]), rtol=1e-4, atol=0.0,
                                            maxiter=500)
    # (at tighter rtol the reference's unscaled breakdown test, chebyshev.cpp:
    # 236-245, stops this fast solve with status -1 first)
    assert info == 0 and its < 60
    np.testing.assert_allclose(x, np.linalg.solve(S, r), rtol=1e-4, atol=1e-4)
    lo, hi, dmin, dmax = orc.gershgorin(d, i, p)
    assert (lo, hi, dmin, dmax) == (0.0, 8.0, 4.0, 4.0)


def test_weighted_ranges_match_the_reference_compiled_from_source(orc):
    """The oracle restates the reference's nnz-weighted partition; where the
    reference checkout is present, its own src/common/cpu_parallel.cpp is
    compiled (oracle/_ref, `make -C oracle ref`) and the two must agree."""
    if orc.build_ref() is None:
        pytest.skip("reference checkout not present")
    rng = np.random.default_rng(11)
    cases = [np.ones(100, np.int64), np.arange(1, 1000, dtype=np.int64), rng.integers(0, 50, 5000),
             np.zeros(10, np.int64), np.asarray([10 ** 6] + [1] * 999, np.int64),
             np.diff(wl.power_law(20000, 3)[0][2]).astype(np.int64)]
    for work in cases:
        for parts in (1, 2, 3, 7, 16, 64):
            assert orc.weighted_ranges(work, parts) == orc.ref_weighted_ranges(work, parts), (work[:5], parts)
