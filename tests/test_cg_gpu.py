"""CG / Jacobi-PCG parity: the device solve vs the CPU oracle (same recurrence).

Bar: same status, iteration count within +-2, solution within the reference
tests' tolerances, residual equal to the reported one. On the stencil matrices
the SpMV rows are summed in the reference's order, so iteration counts are
expected to match exactly.
"""

import numpy as np
import pytest
import scipy.sparse as sp
import torch

import workloads as wl

pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def ms():
    import mlx_sparse

    return mlx_sparse


def _csr(ms, d, i, p, shape):
    return ms.csr_array((_dev(d), _dev(i), _dev(p)), shape=shape, canonical=True)


@pytest.mark.parametrize("name", ["pcg_2x2", "pcg_4x4", "pcg_scaled_poisson", "pcg_diag"])
def test_golden_pcg(ms, golden, name):
    c = golden[name]
    A = _csr(ms, np.asarray(c["A"]["data"], np.float32), np.asarray(c["A"]["indices"], np.int32),
             np.asarray(c["A"]["indptr"], np.int32), c["A"]["shape"])
    b = _dev(np.asarray(c["b"], np.float32))
    x, info = ms.linalg.cg(A, b, M=ms.linalg.preconditioners.jacobi(A), rtol=c["rtol"], atol=c["atol"],
                           maxiter=c["maxiter"], return_info=True)
    assert info.status == 0
    tol = c.get("x_tol", 1e-4)
    np.testing.assert_allclose(x.cpu().numpy(), c["x"], rtol=tol, atol=tol)
    if "max_iterations" in c:
        assert info.iterations <= c["max_iterations"]
        dense = A.todense().cpu().numpy()
        assert info.residual_norm == pytest.approx(
            np.linalg.norm(dense @ x.cpu().numpy() - np.asarray(c["b"], np.float32)), abs=1e-4)


@pytest.mark.parametrize("precond", [False, True])
@pytest.mark.parametrize("make", [lambda: wl.lap2d(48), lambda: wl.poisson3d(16),
                                  lambda: wl.poisson3d(20, np.int64)], ids=["lap2d", "p3d", "p3d_i64"])
def test_parity_with_oracle(ms, orc, precond, make):
    (d, i, p), shape = make()
    n = shape[0]
    xs = wl.uniform_vector(n, 1)
    b = orc.csr_matvec(d, i, p, xs, n)
    A = _csr(ms, d, i, p, shape)
    x0 = np.zeros(n, np.float32)
    if precond:
        inv = np.full(n, 1.0 / float(d.max()), np.float32)
        xr, info_r, res_r, its_r = orc.csr_pcg_jacobi(d, i, p, b, x0, inv, rtol=1e-6, atol=0.0, maxiter=2000)
        M = ms.linalg.preconditioners.jacobi(A)
    else:
        xr, info_r, res_r, its_r = orc.csr_cg(d, i, p, b, x0, rtol=1e-6, atol=0.0, maxiter=2000)
        M = None
    x, info = ms.linalg.cg(A, _dev(b), M=M, rtol=1e-6, maxiter=2000, return_info=True)
    # the reference's breakdown test is not scale-aware, so some of these
    # stop with status -1 near convergence; the device must agree
    assert info.status == info_r
    assert abs(info.iterations - its_r) <= 2
    np.testing.assert_allclose(x.cpu().numpy(), xr, rtol=1e-3, atol=1e-3)
    assert info.residual_norm == pytest.approx(res_r, rel=0.05)


def test_plain_cg_matches_dense_solve(ms):
    (d, i, p), shape = wl.lap2d(12)
    Ad = sp.csr_matrix((d, i, p), shape=shape).toarray().astype(np.float64)
    b = wl.uniform_vector(shape[0], 3)
    x, info = ms.linalg.cg(_csr(ms, d, i, p, shape), _dev(b), rtol=1e-6)
    assert info == 0
    np.testing.assert_allclose(x.cpu().numpy(), np.linalg.solve(Ad, b), rtol=1e-4, atol=1e-4)


def test_status_codes_match_oracle(ms, orc):
    (d, i, p), shape = wl.lap2d(10)
    n = shape[0]
    A = _csr(ms, d, i, p, shape)
    b = wl.uniform_vector(n, 1)
    x0 = np.zeros(n, np.float32)
    # iteration budget exhausted
    _, info = ms.linalg.cg(A, _dev(b), rtol=1e-12, maxiter=3, return_info=True)
    _, info_r, res_r, its_r = orc.csr_cg(d, i, p, b, x0, rtol=1e-12, atol=0.0, maxiter=3)
    assert info.status == info_r == 3 and info.iterations == its_r == 3
    # maxiter == 0 -> status 1
    _, info = ms.linalg.cg(A, _dev(b), maxiter=0, return_info=True)
    assert info.status == 1 and info.iterations == 0
    # non-finite right-hand side -> -3
    bad = b.copy()
    bad[3] = np.inf
    _, info = ms.linalg.cg(A, _dev(bad), maxiter=10, return_info=True)
    assert info.status == -3
    # non-positive preconditioned product -> -2
    M = ms.linalg.preconditioners.diagonal(np.full(n, -4.0, np.float32))
    _, info = ms.linalg.cg(A, _dev(b), M=M, maxiter=10, return_info=True)
    assert info.status == -2
    # already converged (b = 0) -> 0 iterations
    x, info = ms.linalg.cg(A, torch.zeros(n, device="cuda"), return_info=True)
    assert info.status == 0 and info.iterations == 0


def test_split_row_matrix(ms, orc):
    # an SPD matrix with one dense row/column (longer than the CTA bin, so it
    # is cut into chunks) exercises the unfused SpMV + fixup + dot path
    n = 10000
    rng = np.random.default_rng(3)
    M = sp.random(n, n, density=0.0003, random_state=rng, dtype=np.float32)
    M = M + M.T
    M = M.tolil()
    M[5000, :] = 0.001
    M[:, 5000] = 0.001
    M = (M + sp.identity(n, dtype=np.float32) * 8.0).tocsr()
    M.sort_indices()
    d, i, p = M.data.astype(np.float32), M.indices.astype(np.int32), M.indptr.astype(np.int32)
    A = _csr(ms, d, i, p, (n, n))
    assert A.spmv_plan().n_long > 0
    b = wl.uniform_vector(n, 2)
    x, info = ms.linalg.cg(A, _dev(b), rtol=1e-6, maxiter=500, return_info=True)
    xr, info_r, _, its_r = orc.csr_cg(d, i, p, b, np.zeros(n, np.float32), rtol=1e-6, atol=0.0, maxiter=500)
    assert info.status == info_r == 0 and abs(info.iterations - its_r) <= 2
    np.testing.assert_allclose(x.cpu().numpy(), xr, rtol=1e-3, atol=1e-4)


def test_diagonal_sums_duplicates(ms):
    d = np.array([1.0, 2.0, 3.0, 4.0, 5.0], np.float32)
    i = np.array([0, 0, 1, 1, 0], np.int32)
    p = np.array([0, 2, 4, 5], np.int32)
    A = ms.csr_array((_dev(d), _dev(i), _dev(p)), shape=(3, 2))
    assert A.diagonal().cpu().tolist() == [3.0, 7.0]


def test_cached_context_matches_stateless_solve(ms, orc):
    """linalg.cg reuses the matrix's persistent solver; repeated solves (with
    different right-hand sides and a warm start) must give the stateless
    entry point's results bit for bit."""
    from mlx_sparse import _native

    (d, i, p), shape = wl.poisson3d(24)
    n = shape[0]
    A = _csr(ms, d, i, p, shape)
    M = ms.linalg.preconditioners.jacobi(A)
    inv = M.inverse_diagonal.cuda()
    for seed in (1, 2):
        b = _dev(wl.uniform_vector(n, seed))
        x0 = torch.zeros(n, device="cuda") if seed == 1 else b * 0.1
        x, info = ms.linalg.cg(A, b, x0=x0, M=M, rtol=1e-6, maxiter=500, return_info=True)
        xs, info_s, res_s, its_s = _native.csr_pcg_jacobi(A.data, A.indices, A.indptr, b, x0, inv, shape,
                                                          rtol=1e-6, atol=0.0, maxiter=500)
        assert torch.equal(x, xs)
        assert info.status == info_s and info.iterations == its_s
    assert len(A._solvers) == 1


@pytest.mark.parametrize("grid", ["64", "256"])
def test_baseline_pcg_poisson3d(ms, orc, grid):
    """BASELINE config 4 (256^3, and the 64^3 grid of the same recipe): the
    device solve against the oracle's committed result in
    tests/golden/pcg_poisson3d.json - same status, iterations within +-2,
    the first entries of x, and a true relative residual within the target."""
    import json
    import os

    with open(os.path.join(os.path.dirname(__file__), "golden", "pcg_poisson3d.json")) as f:
        g = json.load(f)[grid]
    (d, i, p), shape = wl.poisson3d(g["grid"])
    n = shape[0]
    b = orc.csr_matvec(d, i, p, wl.uniform_vector(n, 1), n, workers=8)
    assert float(np.linalg.norm(b.astype(np.float64))) == pytest.approx(g["b_norm"], rel=1e-9)
    A = _csr(ms, d, i, p, shape)
    bd = _dev(b)
    x, info = ms.linalg.cg(A, bd, M=ms.linalg.preconditioners.jacobi(A), rtol=1e-6, maxiter=2000,
                           return_info=True)
    assert info.status == g["info"] == 0
    assert abs(info.iterations - g["iterations"]) <= 2, (info.iterations, g["iterations"])
    np.testing.assert_allclose(x[:8].cpu().numpy(), g["x_head"], rtol=1e-4, atol=1e-4)
    r = (bd.double() - (A @ x).double()).norm().item()
    assert r <= 1.05e-6 * g["b_norm"], r / g["b_norm"]
