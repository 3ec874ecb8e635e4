"""The DLPack boundary on the GPU: the msx_dl_* entry points (what the
Python layer calls for csr_matvec, csr_matmul, csr_matmat, csr_cg and
csr_pcg_jacobi) give the raw-pointer entry points' results and refuse
tensors they cannot take, with the reference's error kinds."""

import ctypes

import numpy as np
import pytest
import torch

import workloads as wl

pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.fixture(scope="module")
def nat():
    from mlx_sparse import _native

    return _native


def test_dlpack_and_raw_entry_points_agree(nat, orc):
    (d, i, p), shape = wl.ragged_csr(3000, 2000, 4, 30)
    A = [_dev(d), _dev(i), _dev(p)]
    x = _dev(wl.uniform_vector(shape[1], 1))
    y_dl = nat.csr_matvec(*A, x, shape)
    L = nat.extension()
    y_raw = torch.empty_like(y_dl)
    nat.check(L.msx_csr_matvec(0, 0, A[0].data_ptr(), A[1].data_ptr(), A[2].data_ptr(), A[0].numel(),
                               x.data_ptr(), y_raw.data_ptr(), shape[0], shape[1], None,
                               torch.cuda.current_stream().cuda_stream))
    assert torch.equal(y_dl, y_raw)
    B = _dev(wl.uniform_matrix(shape[1], 8, 2))
    np.testing.assert_array_equal(nat.csr_matmul(*A, B, shape).cpu().numpy(),
                                  orc.csr_matmul(d, i, p, B.cpu().numpy(), shape[0]))


def test_dlpack_honours_storage_offsets(nat):
    (d, i, p), shape = wl.lap2d(20)
    A = [_dev(d), _dev(i), _dev(p)]
    big = torch.arange(shape[1] + 7, dtype=torch.float32, device="cuda")
    x = big[7:]  # a view 28 bytes into its storage
    assert torch.equal(nat.csr_matvec(*A, x, shape), nat.csr_matvec(*A, x.clone(), shape))


def test_dlpack_rejections(nat):
    L = nat.extension()
    (d, i, p), shape = wl.lap2d(8)
    A = [_dev(d), _dev(i), _dev(p)]
    x = _dev(wl.uniform_vector(shape[1], 1))
    y = torch.empty(shape[0], device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    dl = nat._DL()
    # non-contiguous x
    xs = torch.zeros(2 * shape[1], device="cuda")[::2]
    assert L.msx_dl_csr_matvec(dl(A[0]), dl(A[1]), dl(A[2]), dl(xs), dl(y), shape[0], shape[1], None, s) == 1
    assert b"contiguous" in L.msx_last_error()
    # indices and indptr of different index dtypes -> TypeError
    assert L.msx_dl_csr_matvec(dl(A[0]), dl(A[1]), dl(A[2].long()), dl(x), dl(y), shape[0], shape[1], None, s) == 2
    # x of the wrong length -> ValueError
    assert L.msx_dl_csr_matvec(dl(A[0]), dl(A[1]), dl(A[2]), dl(x[:-1]), dl(y), shape[0], shape[1], None, s) == 1
    # x of another dtype -> TypeError
    assert L.msx_dl_csr_matvec(dl(A[0]), dl(A[1]), dl(A[2]), dl(x.half()), dl(y), shape[0], shape[1], None, s) == 2
    # a host tensor -> ValueError (no CPU fallback)
    assert L.msx_dl_csr_matvec(dl(A[0]), dl(A[1]), dl(A[2]), dl(x.cpu()), dl(y), shape[0], shape[1], None, s) == 1
    assert b"no CPU fallback" in L.msx_last_error()


def test_dlpack_spgemm_and_solvers(ms_mod, orc):
    ms = ms_mod
    (d, i, p), shape = wl.random_k_per_row(400, 400, 5, 3)
    A = ms.csr_array((_dev(d), _dev(i), _dev(p)), shape=shape, canonical=True)
    C = A @ A
    rd, ri, rp = orc.csr_matmat((d, i, p), (d, i, p), shape, shape)
    np.testing.assert_array_equal(C.indptr.cpu().numpy(), rp)
    np.testing.assert_array_equal(C.indices.cpu().numpy(), ri)
    from mlx_sparse import _native

    (d, i, p), shape = wl.poisson3d(10)
    b = _dev(wl.uniform_vector(shape[0], 1))
    x0 = torch.zeros(shape[0], device="cuda")
    args = (_dev(d), _dev(i), _dev(p))
    x, info, _, its = _native.csr_cg(*args, b, x0, shape, rtol=1e-6, atol=0.0, maxiter=500)
    xr, info_r, _, its_r = orc.csr_cg(d, i, p, b.cpu().numpy(), np.zeros(shape[0], np.float32), rtol=1e-6, atol=0.0,
                                      maxiter=500)
    assert info == info_r and abs(its - its_r) <= 2
    inv = torch.full((shape[0],), 1.0 / 6.0, device="cuda")
    x, info, _, its = _native.csr_pcg_jacobi(*args, b, x0, inv, shape, rtol=1e-6, atol=0.0, maxiter=500)
    xr, info_r, _, its_r = orc.csr_pcg_jacobi(d, i, p, b.cpu().numpy(), np.zeros(shape[0], np.float32),
                                              np.full(shape[0], 1.0 / 6.0, np.float32), rtol=1e-6, atol=0.0,
                                              maxiter=500)
    assert info == info_r and abs(its - its_r) <= 2


@pytest.fixture(scope="module")
def ms_mod():
    import mlx_sparse

    return mlx_sparse
