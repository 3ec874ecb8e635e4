"""COO entry, transposition and the backward products on the GPU (through
the C ABI) against the CPU oracle, and autograd against dense gradients.

Bars: conversions and structures bit-exact (indptr, indices, the source
permutation, the gathered values); matrix products (COO @ B, A^T @ B)
bit-exact in fp32, since every output element sums its entries in the
reference's order; vector products (COO @ x, A^T @ x) within 1e-5 of the row
scale sum |a x|, since rows longer than one lane's share are summed by a
shuffle tree; bf16 within 1e-2; the data cotangents bit-exact in fp32;
autograd within 1e-5 of the dense gradient (the reference's
tests/test_grad.py bound).
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


def _close_rows(y, y_ref, scale, tol=1e-5):
    err = np.abs(y.astype(np.float64) - y_ref.astype(np.float64))
    assert np.all(err <= tol * np.maximum(np.abs(y_ref), scale) + 1e-30), float(np.max(err / (scale + 1e-30)))


def _random_coo(n_rows, n_cols, nnz, seed, it=np.int32, hot_rows=()):
    """Unsorted COO with duplicates; `hot_rows` get many extra entries (to
    reach the CTA and multi-CTA row sorts)."""
    rng = np.random.default_rng(seed)
    row = rng.integers(0, n_rows, nnz)
    col = rng.integers(0, n_cols, nnz)
    extra_r, extra_c = [], []
    for r, cnt in hot_rows:
        extra_r.append(np.full(cnt, r))
        extra_c.append(rng.integers(0, n_cols, cnt))
    if extra_r:
        row = np.concatenate([row] + extra_r)
        col = np.concatenate([col] + extra_c)
        order = rng.permutation(row.size)
        row, col = row[order], col[order]
    dup = rng.integers(0, row.size, row.size // 10)  # exact duplicate coordinates
    row = np.concatenate([row, row[dup]])
    col = np.concatenate([col, col[dup]])
    data = rng.standard_normal(row.size).astype(np.float32)
    return data, row.astype(it), col.astype(it)


@pytest.mark.parametrize("name", ["coo_tocsr_sort", "coo_canonical_dups", "coo_empty"])
def test_golden_coo_tocsr(ms, golden, name):
    c = golden[name]
    A = ms.coo_array((_dev(np.asarray(c["data"], np.float32)), (_dev(np.asarray(c["row"], np.int32)),
                                                                 _dev(np.asarray(c["col"], np.int32)))),
                     shape=c["shape"])
    csr = A.tocsr(canonical=(name == "coo_canonical_dups"))
    assert csr.sorted_indices
    assert csr.indptr.cpu().tolist() == c["indptr"]
    assert csr.indices.cpu().tolist() == c["indices"]
    np.testing.assert_allclose(csr.data.cpu().numpy(), c["out_data"])


@pytest.mark.parametrize("it", [np.int32, np.int64])
@pytest.mark.parametrize("sort_columns", [True, False])
def test_coo_tocsr_matches_oracle(ms, orc, it, sort_columns):
    from mlx_sparse import _native

    # rows of 1, <= 32, <= 2048 and > 2048 entries (all three sort paths)
    data, row, col = _random_coo(3000, 5000, 40000, 1, it, hot_rows=((7, 500), (11, 3000), (2999, 20000)))
    d, i, p, perm = _native.coo_tocsr(_dev(data), _dev(row), _dev(col), (3000, 5000), sort_columns=sort_columns,
                                      with_perm=True)
    rd, ri, rp, rperm = orc.coo_tocsr(data, row, col, 3000, sort_columns=sort_columns)
    np.testing.assert_array_equal(p.cpu().numpy(), rp)
    np.testing.assert_array_equal(i.cpu().numpy(), ri)
    np.testing.assert_array_equal(perm.cpu().numpy(), rperm)
    np.testing.assert_array_equal(d.cpu().numpy(), rd)


def test_coo_tocsr_rejects_out_of_range(ms):
    from mlx_sparse import _native

    with pytest.raises(ValueError, match="inside the matrix shape"):
        _native.coo_tocsr(_dev(np.ones(2, np.float32)), _dev(np.array([0, 3], np.int32)),
                          _dev(np.array([0, 1], np.int32)), (3, 3))


@pytest.mark.parametrize("it", [np.int32, np.int64])
def test_coo_products_match_oracle(ms, orc, it):
    data, row, col = _random_coo(2000, 1500, 30000, 2, it, hot_rows=((5, 4000),))
    A = ms.coo_array((_dev(data), (_dev(row), _dev(col))), shape=(2000, 1500))
    x = wl.uniform_vector(1500, 3)
    B = wl.uniform_matrix(1500, 24, 4)
    scale = orc.coo_matmul(np.abs(data), row, col, np.abs(x), 2000)
    _close_rows((A @ _dev(x)).cpu().numpy(), orc.coo_matmul(data, row, col, x, 2000), scale)
    np.testing.assert_array_equal((A @ _dev(B)).cpu().numpy(), orc.coo_matmul(data, row, col, B, 2000))
    # bf16: fp32 accumulation, one rounding at the store
    Ab = ms.coo_array((_dev(data).bfloat16(), (_dev(row), _dev(col))), shape=(2000, 1500))
    Yb = (Ab @ _dev(B).bfloat16()).float().cpu().numpy()
    Yr = orc.bf16_bits_to_f32(orc.coo_matmul(orc.f32_to_bf16_bits(data), row, col, orc.f32_to_bf16_bits(B), 2000,
                                             bf16=True))
    np.testing.assert_allclose(Yb, Yr, rtol=1e-2, atol=1e-2)


def test_coo_sparse_product_returns_canonical_coo(ms):
    import scipy.sparse as sp

    data, row, col = _random_coo(300, 300, 2000, 5)
    A = ms.coo_array((_dev(data), (_dev(row), _dev(col))), shape=(300, 300))
    C = A @ A
    assert isinstance(C, ms.COOArray)
    S = sp.coo_matrix((data, (row, col)), shape=(300, 300)).tocsr()
    ref = (S @ S).toarray()
    np.testing.assert_allclose(C.todense().cpu().numpy(), ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("it", [np.int32, np.int64])
def test_transpose_structure_and_products(ms, orc, it):
    import scipy.sparse as sp

    from mlx_sparse import _native

    (d, i, p), shape = wl.ragged_csr(3000, 2200, 6, 60, it)
    A = ms.csr_array((_dev(d), _dev(i), _dev(p)), shape=shape, canonical=True)
    T = A.transpose()
    S = sp.csr_matrix((d, i, p), shape=shape).T.tocsr()
    S.sort_indices()
    np.testing.assert_array_equal(T.indptr.cpu().numpy(), S.indptr)
    np.testing.assert_array_equal(T.indices.cpu().numpy(), S.indices)
    np.testing.assert_array_equal(T.data.cpu().numpy(), S.data)
    x = wl.uniform_vector(shape[0], 7)
    B = wl.uniform_matrix(shape[0], 16, 8)
    y_ref = orc.csr_matmul_transpose(d, i, p, x, shape[1])
    Y_ref = orc.csr_matmul_transpose(d, i, p, B, shape[1])
    scale = orc.csr_matmul_transpose(np.abs(d), i, p, np.abs(x), shape[1])
    _close_rows(ms.csr_matvec_transpose(A, _dev(x)).cpu().numpy(), y_ref, scale)
    np.testing.assert_array_equal(ms.csr_matmul_transpose(A, _dev(B)).cpu().numpy(), Y_ref)
    # the stateless C-ABI entry points (transposed structure built per call)
    _close_rows(_native.csr_matvec_transpose(A.data, A.indices, A.indptr, _dev(x), shape).cpu().numpy(), y_ref,
                scale)
    np.testing.assert_array_equal(_native.csr_matmul_transpose(A.data, A.indices, A.indptr, _dev(B), shape)
                                  .cpu().numpy(), Y_ref)


@pytest.mark.parametrize("k", [None, 1, 5, 64])
def test_data_vjp_matches_oracle(ms, orc, k):
    (d, i, p), shape = wl.ragged_csr(2500, 1800, 9, 50)
    A = ms.csr_array((_dev(d), _dev(i), _dev(p)), shape=shape, canonical=True)
    if k is None:
        x, cot = wl.uniform_vector(shape[1], 1), wl.uniform_vector(shape[0], 2)
        got = ms.csr_matvec_data_vjp(A, _dev(x), _dev(cot))
    else:
        x, cot = wl.uniform_matrix(shape[1], k, 1), wl.uniform_matrix(shape[0], k, 2)
        got = ms.csr_matmul_data_vjp(A, _dev(x), _dev(cot))
    np.testing.assert_array_equal(got.cpu().numpy(), orc.csr_data_vjp(i, p, x, cot))


def test_golden_gradients(ms, golden):
    c = golden["grad_csr_matvec"]
    data = _dev(np.asarray(c["A"]["data"], np.float32)).requires_grad_()
    A = ms.csr_array((data, _dev(np.asarray(c["A"]["indices"], np.int32)),
                      _dev(np.asarray(c["A"]["indptr"], np.int32))), shape=c["A"]["shape"], canonical=True)
    x = _dev(np.asarray(c["x"], np.float32)).requires_grad_()
    ((A @ x) ** 2).sum().backward()
    np.testing.assert_allclose(data.grad.cpu().numpy(), c["grad_data"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(x.grad.cpu().numpy(), c["grad_x"], rtol=1e-5, atol=1e-5)

    c = golden["grad_coo_matmul"]
    data = _dev(np.asarray(c["data"], np.float32)).requires_grad_()
    A = ms.coo_array((data, (_dev(np.asarray(c["row"], np.int32)), _dev(np.asarray(c["col"], np.int32)))),
                     shape=c["shape"])
    B = _dev(np.asarray(c["B"], np.float32)).requires_grad_()
    ((A @ B) ** 2).sum().backward()
    np.testing.assert_allclose(data.grad.cpu().numpy(), c["grad_data"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(B.grad.cpu().numpy(), c["grad_B"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("rank", [1, 2])
def test_autograd_matches_dense(ms, rank):
    (d, i, p), shape = wl.ragged_csr(700, 500, 3, 30)
    data = _dev(d).requires_grad_()
    A = ms.csr_array((data, _dev(i), _dev(p)), shape=shape, canonical=True)
    rhs = _dev(wl.uniform_vector(shape[1], 4) if rank == 1 else wl.uniform_matrix(shape[1], 6, 4)).requires_grad_()
    w = _dev(wl.uniform_vector(shape[0], 5) if rank == 1 else wl.uniform_matrix(shape[0], 6, 5))
    ((A @ rhs) * w).sum().backward()
    # dense float64 reference on the CPU
    rows = np.repeat(np.arange(shape[0]), np.diff(p))
    dd = torch.tensor(d, dtype=torch.float64, requires_grad=True)
    dense = torch.zeros(shape, dtype=torch.float64).index_put((torch.tensor(rows), torch.tensor(i, dtype=torch.long)),
                                                              dd, accumulate=True)
    r64 = rhs.detach().cpu().double().requires_grad_()
    ((dense @ r64) * w.cpu().double()).sum().backward()
    np.testing.assert_allclose(data.grad.cpu().numpy(), dd.grad.numpy(), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(rhs.grad.cpu().numpy(), r64.grad.numpy(), rtol=1e-5, atol=1e-5)
