"""SpMV parity: CUDA path (through the C ABI) vs the CPU oracle.

Tolerance (fp32): per row |y - y_ref| <= 1e-5 * max(|y_ref|, sum_j |a_ij x_j|),
the north-star's 1e-5 relative per-row bound made safe for rows that cancel;
fp16/bf16 (fp32 accumulation): 1e-2 of the same scale.
"""

import os

import numpy as np
import pytest
import torch

import workloads as wl

pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _csr(ms, d, i, p, shape, dtype=torch.float32):
    return ms.csr_array((_dev(d).to(dtype), _dev(i), _dev(p)), shape=shape, canonical=True)


def _row_scale(orc, d, i, p, x, n):
    return np.maximum(np.abs(orc.csr_matvec(np.abs(d), i, p, np.abs(x), n, workers=8)), 1e-30)


def _check(y, y_ref, scale, tol):
    err = np.abs(y.astype(np.float64) - y_ref.astype(np.float64))
    bound = tol * np.maximum(np.abs(y_ref), scale) + 1e-30
    bad = np.nonzero(err > bound)[0]
    assert bad.size == 0, f"{bad.size} rows out of tolerance, first {bad[:5]}, err {err[bad[:5]]}"


@pytest.fixture(scope="module")
def ms():
    import mlx_sparse

    assert torch.cuda.is_available()
    return mlx_sparse


@pytest.mark.parametrize("it", [np.int32, np.int64])
def test_golden(ms, golden, it):
    for name in ("spmv_hand", "spmv_scipy_456"):
        c = golden[name]
        A = _csr(ms, np.asarray(c["A"]["data"], np.float32), np.asarray(c["A"]["indices"], it),
                 np.asarray(c["A"]["indptr"], it), c["A"]["shape"])
        y = (A @ _dev(np.asarray(c["x"], np.float32))).cpu().numpy()
        np.testing.assert_allclose(y, c["y"], rtol=1e-5, atol=1e-5)


CASES = [
    ("lap2d_64", lambda it: wl.lap2d(64, it)),
    ("random_k16", lambda it: wl.random_k_per_row(3000, 2500, 16, 7, it)),
    ("ragged_split_rows", lambda it: wl.ragged_csr(5000, 3000, 9, 40, it)),
    ("power_law_small", lambda it: wl.power_law(20000, 3, it)),
    ("long_rows", lambda it: wl.ragged_csr(300, 60000, 2, 600, it)),
    ("one_long_row", lambda it: _one_row(70000, it)),
]


def _one_row(n_cols, it):
    rng = np.random.default_rng(12)
    cols = np.sort(rng.choice(n_cols, size=n_cols // 2, replace=False))
    return (rng.uniform(-1, 1, cols.size).astype(np.float32), cols.astype(it),
            np.array([0, cols.size], dtype=it)), (1, n_cols)


@pytest.mark.parametrize("it", [np.int32, np.int64])
@pytest.mark.parametrize("name,make", CASES, ids=[c[0] for c in CASES])
def test_parity_fp32(ms, orc, it, name, make):
    (d, i, p), shape = make(it)
    x = wl.uniform_vector(shape[1], 1)
    y_ref = orc.csr_matvec(d, i, p, x, shape[0], workers=8)
    A = _csr(ms, d, i, p, shape)
    y = (A @ _dev(x)).cpu().numpy()
    scale = _row_scale(orc, d, i, p, x, shape[0])
    _check(y, y_ref, scale, 1e-5)
    # the stateless C-ABI call (no plan: merge-path tiles in scratch)
    from mlx_sparse import _native

    y2 = _native.csr_matvec(A.data, A.indices, A.indptr, _dev(x), A.shape).cpu().numpy()
    _check(y2, y_ref, scale, 1e-5)


def test_short_rows_match_reference_order_exactly(ms, orc):
    # Rows of <= 2 thread shares are summed in the reference's order: bit-exact.
    (d, i, p), shape = wl.lap2d(128)
    x = wl.uniform_vector(shape[1], 0)
    y = (_csr(ms, d, i, p, shape) @ _dev(x)).cpu().numpy()
    y_ref = orc.csr_matvec(d, i, p, x, shape[0])
    np.testing.assert_array_equal(y, y_ref)


def test_split_rows_present_and_deterministic(ms, orc):
    # rows of 24,000 nonzeros are cut into 8192-nonzero chunks
    (d, i, p), shape = wl.ragged_csr(2000, 30000, 4, 600)
    A = _csr(ms, d, i, p, shape)
    assert A.spmv_plan().n_long > 0
    x = _dev(wl.uniform_vector(shape[1], 2))
    y1 = (A @ x).cpu().numpy()
    y2 = (A @ x).cpu().numpy()
    np.testing.assert_array_equal(y1, y2)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_types(ms, orc, dtype):
    (d, i, p), shape = wl.ragged_csr(3000, 2000, 5, 25)
    x = wl.uniform_vector(shape[1], 3)
    A = _csr(ms, d, i, p, shape, dtype)
    xt = _dev(x).to(dtype)
    y = (A @ xt).float().cpu().numpy()
    if dtype == torch.float16:
        y_ref = orc.csr_matvec(d.astype(np.float16), i, p, x.astype(np.float16), shape[0]).astype(np.float32)
    else:
        y_ref = orc.bf16_bits_to_f32(orc.csr_matvec(orc.f32_to_bf16_bits(d), i, p, orc.f32_to_bf16_bits(x),
                                                    shape[0], bf16=True))
    _check(y, y_ref, _row_scale(orc, d, i, p, x, shape[0]), 1e-2)


def test_edge_cases(ms):
    # empty matrix, rows without nonzeros, nnz == 0
    A = ms.csr_array((torch.zeros(0, device="cuda"), torch.zeros(0, dtype=torch.int32, device="cuda"),
                      torch.zeros(1, dtype=torch.int32, device="cuda")), shape=(0, 5))
    assert (A @ torch.ones(5, device="cuda")).shape == (0,)
    A = ms.csr_array((torch.zeros(0, device="cuda"), torch.zeros(0, dtype=torch.int32, device="cuda"),
                      torch.zeros(7, dtype=torch.int32, device="cuda")), shape=(6, 5))
    y = A @ torch.ones(5, device="cuda")
    assert torch.equal(y, torch.zeros(6, device="cuda"))
    # leading/trailing empty rows around a single entry
    A = ms.csr_array((torch.tensor([2.0], device="cuda"), torch.tensor([1], dtype=torch.int32, device="cuda"),
                      torch.tensor([0, 0, 0, 1, 1, 1], dtype=torch.int32, device="cuda")), shape=(5, 3))
    y = A @ torch.tensor([1.0, 3.0, 5.0], device="cuda")
    assert y.cpu().tolist() == [0.0, 0.0, 6.0, 0.0, 0.0]


def test_non_contiguous_inputs(ms):
    (d, i, p), shape = wl.lap2d(16)
    A = _csr(ms, d, i, p, shape)
    x_full = torch.arange(2 * shape[1], dtype=torch.float32, device="cuda")
    x = x_full[::2]
    np.testing.assert_allclose((A @ x).cpu().numpy(), (A @ x.contiguous()).cpu().numpy())


def test_full_size_lap2d(ms, orc):
    (d, i, p), shape = wl.lap2d(1024)
    x = wl.uniform_vector(shape[1], 0)
    y = (_csr(ms, d, i, p, shape) @ _dev(x)).cpu().numpy()
    y_ref = orc.csr_matvec(d, i, p, x, shape[0], workers=8)
    _check(y, y_ref, _row_scale(orc, d, i, p, x, shape[0]), 1e-5)


def test_full_size_power_law_int64(ms, orc):
    """BASELINE config 3 at full size: 4,194,304 rows, int64 indices,
    Lomax(2.1) row lengths (mean ~20), per-row 1e-5."""
    (d, i, p), shape = wl.power_law(1 << 22, 3, np.int64)
    x = wl.uniform_vector(shape[1], 5)
    A = _csr(ms, d, i, p, shape)
    xd = _dev(x)
    y = (A @ xd).cpu().numpy()
    y_ref = orc.csr_matvec(d, i, p, x, shape[0], workers=8)
    scale = _row_scale(orc, d, i, p, x, shape[0])
    _check(y, y_ref, scale, 1e-5)
    from mlx_sparse import _native

    y2 = _native.csr_matvec(A.data, A.indices, A.indptr, xd, A.shape).cpu().numpy()
    _check(y2, y_ref, scale, 1e-5)


@pytest.fixture
def tma_pipeline():
    """Selects the opt-in TMA bulk-copy pipeline of the stateless tile SpMV
    (read at every call) for one test."""
    old = os.environ.get("MSX_SPMV_TMA")
    os.environ["MSX_SPMV_TMA"] = "1"
    yield
    if old is None:
        del os.environ["MSX_SPMV_TMA"]
    else:
        os.environ["MSX_SPMV_TMA"] = old


def test_tma_pipeline_matches_plain_loads(ms, orc):
    from mlx_sparse import _native

    (d, i, p), shape = wl.ragged_csr(30000, 20000, 9, 300)
    A = _csr(ms, d, i, p, shape)
    x = _dev(wl.uniform_vector(shape[1], 3))
    y_plain = _native.csr_matvec(A.data, A.indices, A.indptr, x, A.shape)
    os.environ["MSX_SPMV_TMA"] = "1"
    try:
        y_tma = _native.csr_matvec(A.data, A.indices, A.indptr, x, A.shape)
        _native.check_device_errors()
    finally:
        del os.environ["MSX_SPMV_TMA"]
    assert torch.equal(y_plain, y_tma)
    xh = wl.uniform_vector(shape[1], 3)
    y_ref = orc.csr_matvec(d, i, p, xh, shape[0])
    _check(y_plain.cpu().numpy(), y_ref, _row_scale(orc, d, i, p, xh, shape[0]), 1e-5)


def test_bulk_copy_wait_timeout_is_reported(ms, tma_pipeline):
    """A bulk-copy wait that gives up is reported by msx_check_device_errors
    (the poll limit is set to 0 so every wait gives up at once; the copies
    still land and are waited for before the kernel exits)."""
    from mlx_sparse import _native

    L = _native.extension()
    (d, i, p), shape = wl.ragged_csr(4000, 3000, 7, 40)
    A = _csr(ms, d, i, p, shape)
    x = _dev(wl.uniform_vector(shape[1], 1))
    stream = torch.cuda.current_stream().cuda_stream
    _native.check(L.msx_check_device_errors(stream))
    y_ok = _native.csr_matvec(A.data, A.indices, A.indptr, x, A.shape)
    try:
        _native.check(L.msx_debug_set_spmv_poll_limit(0))
        _native.csr_matvec(A.data, A.indices, A.indptr, x, A.shape)
        assert L.msx_check_device_errors(stream) == 4
        assert b"gave up" in L.msx_last_error()
    finally:
        _native.check(L.msx_debug_set_spmv_poll_limit(-1))
    # the flag was cleared by the check; the next call is whole again
    y = _native.csr_matvec(A.data, A.indices, A.indptr, x, A.shape)
    _native.check(L.msx_check_device_errors(stream))
    assert torch.equal(y, y_ok)
