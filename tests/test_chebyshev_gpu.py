"""Chebyshev and diagonal preconditioners on the GPU against the CPU oracle.

Bars: the preconditioner applications and the Gershgorin bounds bit-exact
(every element follows the reference's float arithmetic and summation
order); Chebyshev-PCG: same status as the oracle, iterations within +-2,
solution within 1e-3 (the Jacobi-PCG bar).
"""

import numpy as np
import pytest
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


def _dense(d, i, p, shape):
    import scipy.sparse as sp

    return sp.csr_matrix((d, i, p), shape=shape).toarray().astype(np.float64)


def _shifted_poisson(m, shift, it=np.int32):
    (d, i, p), shape = wl.poisson3d(m, it)
    rows = np.repeat(np.arange(shape[0]), np.diff(p))
    d = d.copy()
    d[i.astype(np.int64) == rows] += np.float32(shift)
    return (d, i, p), shape


@pytest.mark.parametrize("k", [None, 3])
def test_diagonal_apply_is_exact(ms, k):
    inv = wl.uniform_vector(1000, 1)
    rhs = wl.uniform_vector(1000, 2) if k is None else wl.uniform_matrix(1000, k, 2)
    M = ms.linalg.preconditioners.diagonal(_dev(inv), inverse=True)
    got = M.solve(_dev(rhs)).cpu().numpy()
    ref = inv * rhs if k is None else inv[:, None] * rhs
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("it", [np.int32, np.int64])
@pytest.mark.parametrize("degree", [1, 2, 3, 5])
@pytest.mark.parametrize("k", [None, 4])
def test_chebyshev_apply_matches_oracle(ms, orc, it, degree, k):
    (d, i, p), shape = _shifted_poisson(12, 0.5, it)
    rhs = wl.uniform_vector(shape[0], 3) if k is None else wl.uniform_matrix(shape[0], k, 3)
    M = ms.linalg.preconditioners.ChebyshevPreconditioner(A=_csr(ms, d, i, p, shape), degree=degree,
                                                          lambda_min=0.5, lambda_max=12.5)
    got = M.solve(_dev(rhs)).cpu().numpy()
    ref = orc.chebyshev_apply(d, i, p, rhs, degree=degree, lambda_min=0.5, lambda_max=12.5)
    np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("it", [np.int32, np.int64])
def test_gershgorin_bounds_match_oracle(ms, orc, it):
    from mlx_sparse import _native

    for (d, i, p), shape in (_shifted_poisson(10, 0.25, it), wl.lap2d(30, it)):
        got = _native.csr_gershgorin_bounds(_dev(d), _dev(i), _dev(p), shape)
        assert got == orc.gershgorin(d, i, p)


@pytest.mark.parametrize("degree", [1, 2, 4])
@pytest.mark.parametrize("make", [lambda: _shifted_poisson(16, 0.0), lambda: wl.lap2d(40),
                                  lambda: _shifted_poisson(14, 0.0, np.int64)], ids=["p3d", "lap2d", "p3d_i64"])
def test_pcg_chebyshev_matches_oracle(ms, orc, degree, make):
    (d, i, p), shape = make()
    n = shape[0]
    b = orc.csr_matvec(d, i, p, wl.uniform_vector(n, 1), n)
    lmin, lmax = 0.05, float(np.max(np.abs(d))) * 2.0
    A = _csr(ms, d, i, p, shape)
    M = ms.linalg.preconditioners.ChebyshevPreconditioner(A=A, degree=degree, lambda_min=lmin, lambda_max=lmax)
    x, info = ms.linalg.cg(A, _dev(b), M=M, rtol=1e-6, maxiter=2000, return_info=True)
    xr, info_r, res_r, its_r = orc.csr_pcg_chebyshev(d, i, p, b, np.zeros(n, np.float32), (d, i, p), degree=degree,
                                                     lambda_min=lmin, lambda_max=lmax, rtol=1e-6, atol=0.0,
                                                     maxiter=2000)
    assert info.status == info_r
    assert abs(info.iterations - its_r) <= 2, (info.iterations, its_r)
    np.testing.assert_allclose(x.cpu().numpy(), xr, rtol=1e-3, atol=1e-3)


def test_chebyshev_bounds_from_gershgorin_and_lanczos(ms, orc):
    # diagonally dominant: Gershgorin interval; plain Poisson: lower bound 0,
    # so the Lanczos estimate supplies lambda_min
    (d, i, p), shape = _shifted_poisson(10, 1.0)
    M = ms.linalg.preconditioners.chebyshev(_csr(ms, d, i, p, shape), degree=3)
    assert M.spectral_info["lambda_min_source"] == "gershgorin"
    assert M.lambda_min == pytest.approx(1.0) and M.lambda_max == pytest.approx(13.0)
    (d, i, p), shape = wl.poisson3d(10)
    A = _csr(ms, d, i, p, shape)
    M = ms.linalg.preconditioners.chebyshev(A, degree=3)
    assert M.spectral_info["lambda_min_source"] == "lanczos_0.5"
    true_min = 6.0 - 6.0 * np.cos(np.pi / 11)  # smallest eigenvalue of the 10^3 Poisson matrix
    assert 0.0 < M.lambda_min <= true_min
    b = wl.uniform_vector(shape[0], 2)
    x, info = ms.linalg.cg(A, _dev(b), M=M, rtol=1e-5, maxiter=500, return_info=True)
    xr, info_r, _, its_r = orc.csr_pcg_chebyshev(d, i, p, b, np.zeros(shape[0], np.float32), (d, i, p), degree=3,
                                                 lambda_min=M.lambda_min, lambda_max=M.lambda_max, rtol=1e-5,
                                                 atol=0.0, maxiter=500)
    # (the reference's unscaled breakdown test may end such a fast solve with
    # status -1 near convergence; the device must agree with the oracle)
    assert info.status == info_r and abs(info.iterations - its_r) <= 2
    np.testing.assert_allclose(x.cpu().numpy(), xr, rtol=1e-3, atol=1e-3)
    assert np.linalg.norm(xr - np.linalg.solve(_dense(d, i, p, shape), b)) <= 1e-2 * np.linalg.norm(xr)


def test_chebyshev_status_codes(ms, orc):
    (d, i, p), shape = wl.lap2d(10)
    n = shape[0]
    A = _csr(ms, d, i, p, shape)
    M = ms.linalg.preconditioners.ChebyshevPreconditioner(A=A, degree=2, lambda_min=0.1, lambda_max=8.0)
    b = wl.uniform_vector(n, 1)
    _, info = ms.linalg.cg(A, _dev(b), M=M, rtol=1e-12, maxiter=3, return_info=True)
    _, info_r, _, its_r = orc.csr_pcg_chebyshev(d, i, p, b, np.zeros(n, np.float32), (d, i, p), degree=2,
                                                lambda_min=0.1, lambda_max=8.0, rtol=1e-12, atol=0.0, maxiter=3)
    assert info.status == info_r == 3 and info.iterations == its_r == 3
    bad = b.copy()
    bad[5] = np.inf
    _, info = ms.linalg.cg(A, _dev(bad), M=M, maxiter=10, return_info=True)
    assert info.status == -3
    with pytest.raises(ValueError, match="lambda_min"):
        ms.linalg.preconditioners.ChebyshevPreconditioner(A=A, degree=2, lambda_min=2.0, lambda_max=1.0)
