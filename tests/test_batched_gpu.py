"""Batched products (one CSR matrix, a batch of dense vectors or matrices) vs
the CPU oracle applied per batch entry: the reference's batched kernels sum
each output element over its row's nonzeros in order, exactly like the
unbatched ones, so the bound is the SpMV/SpMM one (fp32 rtol = atol = 1e-5,
bf16 3e-2)."""

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


def _csr(ms, d, i, p, shape, dtype=torch.float32):
    return ms.csr_array((_dev(d).to(dtype), _dev(i), _dev(p)), shape=shape, canonical=True)


@pytest.mark.parametrize("batch_shape", [(1,), (3,), (8,), (2, 5), (0,)])
@pytest.mark.parametrize("it", [np.int32, np.int64])
def test_batched_matvec_fp32(ms, orc, batch_shape, it):
    (d, i, p), shape = wl.ragged_csr(1300, 700, 5, 24, it)
    nb = int(np.prod(batch_shape))
    X = wl.uniform_matrix(max(nb, 1), shape[1], 11)[:nb].reshape(*batch_shape, shape[1])
    Y = ms.csr_batched_matvec(_csr(ms, d, i, p, shape), _dev(X)).cpu().numpy()
    assert Y.shape == (*batch_shape, shape[0])
    flat = X.reshape(nb, shape[1])
    ref = np.stack([orc.csr_matvec(d, i, p, flat[b], shape[0]) for b in range(nb)]) if nb else np.zeros(
        (0, shape[0]), np.float32)
    np.testing.assert_allclose(Y.reshape(nb, shape[0]), ref, rtol=1e-5, atol=1e-5)


def test_batched_matvec_bf16(ms, orc):
    (d, i, p), shape = wl.random_k_per_row(900, 600, 12, 3)
    X = wl.uniform_matrix(6, shape[1], 12)
    A = _csr(ms, d, i, p, shape, torch.bfloat16)
    Y = ms.csr_batched_matvec(A, _dev(X).to(torch.bfloat16)).float().cpu().numpy()
    dq = A.data.float().cpu().numpy()
    Xq = _dev(X).to(torch.bfloat16).float().cpu().numpy()
    ref = np.stack([orc.csr_matvec(dq, i, p, Xq[b], shape[0]) for b in range(6)])
    np.testing.assert_allclose(Y, ref, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("batch_shape", [(1,), (4,), (2, 3)])
@pytest.mark.parametrize("k", [1, 5, 16, 64])
def test_batched_matmul_fp32(ms, orc, batch_shape, k):
    (d, i, p), shape = wl.ragged_csr(800, 500, 7, 20)
    nb = int(np.prod(batch_shape))
    B = wl.uniform_matrix(nb * shape[1], k, 13).reshape(*batch_shape, shape[1], k)
    A = _csr(ms, d, i, p, shape)
    Y = ms.csr_batched_matmul(A, _dev(B)).cpu().numpy()
    Y_mm = (A @ _dev(B)).cpu().numpy()  # __matmul__ routes rank >= 3 to the same native call
    assert Y.shape == (*batch_shape, shape[0], k)
    flat = B.reshape(nb, shape[1], k)
    ref = np.stack([orc.csr_matmul(d, i, p, flat[b], shape[0]) for b in range(nb)])
    np.testing.assert_allclose(Y.reshape(nb, shape[0], k), ref, rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(Y, Y_mm)


def test_batched_validation(ms):
    (d, i, p), shape = wl.ragged_csr(50, 40, 1, 6)
    A = _csr(ms, d, i, p, shape)
    with pytest.raises(ValueError, match="rank-2 or higher"):
        ms.csr_batched_matvec(A, torch.zeros(40, device="cuda"))
    with pytest.raises(ValueError, match="n_cols"):
        ms.csr_batched_matvec(A, torch.zeros(3, 41, device="cuda"))
    with pytest.raises(TypeError, match="same dtype"):
        ms.csr_batched_matvec(A, torch.zeros(3, 40, device="cuda", dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="rank-3 or higher"):
        ms.csr_batched_matmul(A, torch.zeros(40, 2, device="cuda"))
    with pytest.raises(ValueError, match="n_cols"):
        ms.csr_batched_matmul(A, torch.zeros(2, 41, 2, device="cuda"))
