"""SpGEMM parity: CUDA path vs the CPU oracle. Structure (indptr, indices) must
be bit-exact; values are accumulated in the reference's order so they are
expected bit-exact too (asserted: rtol 1e-5, atol 1e-6, plus an exact-match
fraction)."""

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


def _csr(ms, d, i, p, shape, dtype=torch.float32, canonical=True):
    return ms.csr_array((_dev(d).to(dtype), _dev(i), _dev(p)), shape=shape, canonical=canonical)


def _compare(C, ref, exact_frac=0.999):
    rd, ri, rp = ref
    np.testing.assert_array_equal(C.indptr.cpu().numpy(), rp)
    np.testing.assert_array_equal(C.indices.cpu().numpy(), ri)
    d = C.data.float().cpu().numpy()
    np.testing.assert_allclose(d, rd, rtol=1e-5, atol=1e-6)
    if d.size:
        assert np.mean(d == rd) >= exact_frac
    assert C.has_canonical_format and C.sorted_indices


@pytest.mark.parametrize("name", ["spgemm_cancel", "spgemm_dense_ordered"])
def test_golden(ms, golden, name):
    c = golden[name]

    def arr(A):
        return (np.asarray(A["data"], np.float32), np.asarray(A["indices"], np.int32),
                np.asarray(A["indptr"], np.int32))

    A = _csr(ms, *arr(c["A"]), c["A"]["shape"])
    B = _csr(ms, *arr(c["B"]), c["B"]["shape"], canonical=False)
    C = A @ B
    np.testing.assert_array_equal(C.indices.cpu().numpy(), c["C"]["indices"])
    np.testing.assert_array_equal(C.indptr.cpu().numpy(), c["C"]["indptr"])
    np.testing.assert_allclose(C.data.cpu().numpy(), c["C"]["data"], rtol=1e-5, atol=1e-6)
    assert np.all(C.data.cpu().numpy() != 0)


@pytest.mark.parametrize("lit,rit", [(np.int32, np.int32), (np.int64, np.int64), (np.int32, np.int64)])
def test_random_parity(ms, orc, lit, rit):
    (ad, ai, ap), sa = wl.random_k_per_row(3000, 2000, 8, 21, lit)
    (bd, bi, bp), sb = wl.random_k_per_row(2000, 2500, 8, 22, rit)
    C = _csr(ms, ad, ai, ap, sa) @ _csr(ms, bd, bi, bp, sb)
    ref = orc.csr_matmat((ad, ai, ap), (bd, bi, bp), sa, sb)
    _compare(C, ref)
    expect = np.int32 if (lit == np.int32 and rit == np.int32) else np.int64
    assert C.indices.cpu().numpy().dtype == expect


def test_all_bins(ms, orc):
    # ragged rows: empty rows, warp-sized, CTA-sized (>256 products) and dense
    # (>4096 products) rows all appear
    (ad, ai, ap), sa = wl.ragged_csr(600, 500, 31, 40)
    (bd, bi, bp), sb = wl.ragged_csr(500, 3000, 32, 30)
    work = np.array([np.sum(np.diff(bp)[ai[ap[r]:ap[r + 1]]]) for r in range(sa[0])])
    assert (work == 0).any() and ((work > 0) & (work <= 256)).any()
    assert ((work > 256) & (work <= 4096)).any() and (work > 4096).any()
    C = _csr(ms, ad, ai, ap, sa) @ _csr(ms, bd, bi, bp, sb)
    _compare(C, orc.csr_matmat((ad, ai, ap), (bd, bi, bp), sa, sb))


def test_exact_cancellation_is_pruned(ms, orc):
    # rows built so that some products cancel exactly
    A = (np.array([1.0, 1.0, 2.0, -2.0], np.float32), np.array([0, 1, 0, 1], np.int32),
         np.array([0, 2, 4], np.int32))
    B = (np.array([3.0, 5.0, -3.0, 7.0], np.float32), np.array([0, 2, 0, 1], np.int32),
         np.array([0, 2, 4], np.int32))
    C = _csr(ms, *A, (2, 2)) @ _csr(ms, *B, (2, 3))
    ref = orc.csr_matmat(A, B, (2, 2), (2, 3))
    _compare(C, ref, exact_frac=1.0)
    assert 0 not in C.data.cpu().numpy()


def test_unsorted_and_duplicate_rhs(ms, orc):
    # rhs rows with unsorted and repeated columns (non-canonical): same result
    rng = np.random.default_rng(5)
    n = 300
    bp = np.arange(0, 6 * n + 1, 6, dtype=np.int32)
    bi = rng.integers(0, 50, 6 * n).astype(np.int32)
    bd = rng.standard_normal(6 * n).astype(np.float32)
    (ad, ai, ap), sa = wl.ragged_csr(200, n, 8, 20)
    C = _csr(ms, ad, ai, ap, sa) @ _csr(ms, bd, bi, bp, (n, 50), canonical=False)
    _compare(C, orc.csr_matmat((ad, ai, ap), (bd, bi, bp), sa, (n, 50)))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_types(ms, orc, dtype):
    (ad, ai, ap), sa = wl.random_k_per_row(800, 800, 6, 3)
    C = _csr(ms, ad, ai, ap, sa, dtype) @ _csr(ms, ad, ai, ap, sa, dtype)
    if dtype == torch.float16:
        ref = orc.csr_matmat((ad.astype(np.float16), ai, ap), (ad.astype(np.float16), ai, ap), sa, sa)
        rd = ref[0].astype(np.float32)
    else:
        b = orc.f32_to_bf16_bits(ad)
        ref = orc.csr_matmat((b, ai, ap), (b, ai, ap), sa, sa, bf16=True)
        rd = orc.bf16_bits_to_f32(ref[0])
    np.testing.assert_array_equal(C.indptr.cpu().numpy(), ref[2])
    np.testing.assert_array_equal(C.indices.cpu().numpy(), ref[1])
    np.testing.assert_allclose(C.data.float().cpu().numpy(), rd, rtol=1e-2, atol=1e-3)


def test_sum_duplicates_via_identity(ms):
    # canonicalize(): sorted rows, duplicates summed in stored order, zeros kept
    d = np.array([1.0, 2.0, -1.0, 4.0, 5.0], np.float32)
    i = np.array([3, 0, 3, 1, 1], np.int32)
    p = np.array([0, 3, 5], np.int32)
    A = _csr(ms, d, i, p, (2, 4), canonical=False).canonicalize()
    assert A.indices.cpu().tolist() == [0, 3, 1]
    assert A.data.cpu().tolist() == [2.0, 0.0, 9.0]
    assert A.indptr.cpu().tolist() == [0, 2, 3]


def test_empty_operands(ms):
    A = ms.csr_array((torch.zeros(0, device="cuda"), torch.zeros(0, dtype=torch.int32, device="cuda"),
                      torch.zeros(4, dtype=torch.int32, device="cuda")), shape=(3, 5))
    C = A @ A.__class__(A.data, A.indices, torch.zeros(6, dtype=torch.int32, device="cuda"), (5, 2))
    assert C.nnz == 0 and C.indptr.cpu().tolist() == [0, 0, 0, 0]


def test_full_size_config(ms, orc):
    (ad, ai, ap), sa = wl.random_k_per_row(1 << 18, 1 << 18, 8, 4)
    A = _csr(ms, ad, ai, ap, sa)
    C = A @ A
    _compare(C, orc.csr_matmat((ad, ai, ap), (ad, ai, ap), sa, sa))


@pytest.mark.parametrize("n_cols", [40, 5000, 1 << 21])
def test_four_rows_per_warp_bin(ms, orc, n_cols):
    # rows of <= 8 lhs entries and <= 64 products, packed four to a warp:
    # ragged lengths, empty lhs and rhs rows, a row count that is not a
    # multiple of four, and few (n_cols 40: many repeated columns) to no
    # repeats
    rng = np.random.default_rng(n_cols)
    m, k = 1001, 700
    alen = rng.integers(0, 9, m)
    blen = rng.integers(0, 9, k)
    ap = np.concatenate([[0], np.cumsum(alen)]).astype(np.int32)
    bp = np.concatenate([[0], np.cumsum(blen)]).astype(np.int32)
    ai = np.concatenate([np.sort(rng.choice(k, n, replace=False)) for n in alen]).astype(np.int32)
    bi = rng.integers(0, n_cols, bp[-1]).astype(np.int32)
    ad = rng.standard_normal(ap[-1]).astype(np.float32)
    bd = rng.standard_normal(bp[-1]).astype(np.float32)
    C = _csr(ms, ad, ai, ap, (m, k)) @ _csr(ms, bd, bi, bp, (k, n_cols), canonical=False)
    _compare(C, orc.csr_matmat((ad, ai, ap), (bd, bi, bp), (m, k), (k, n_cols)), exact_frac=1.0)
