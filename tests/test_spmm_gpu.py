"""SpMM parity: CUDA path vs the CPU oracle.

Every output element is summed over its row's nonzeros in stored order with
separate multiply and add roundings, as the reference does, so fp32 results
are asserted bit-exact; the bound written in the north star (rtol 1e-5 fp32,
1e-2 for fp16/bf16 with fp32 accumulation) is asserted as well.
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


def _csr(ms, d, i, p, shape, dtype=torch.float32):
    return ms.csr_array((_dev(d).to(dtype), _dev(i), _dev(p)), shape=shape, canonical=True)


def test_golden(ms, golden):
    for name in ("spmm_hand", "spmm_scipy_789", "spmm_lowp"):
        c = golden[name]
        A = _csr(ms, np.asarray(c["A"]["data"], np.float32), np.asarray(c["A"]["indices"], np.int32),
                 np.asarray(c["A"]["indptr"], np.int32), c["A"]["shape"])
        Y = (A @ _dev(np.asarray(c["B"], np.float32))).cpu().numpy()
        np.testing.assert_allclose(Y, c["Y"], rtol=1e-5, atol=1e-5)
    c = golden["spmm_lowp"]
    for dtype, tol in ((torch.float16, 5e-3), (torch.bfloat16, 3e-2)):
        A = _csr(ms, np.asarray(c["A"]["data"], np.float32), np.asarray(c["A"]["indices"], np.int32),
                 np.asarray(c["A"]["indptr"], np.int32), c["A"]["shape"], dtype)
        Y = (A @ _dev(np.asarray(c["B"], np.float32)).to(dtype)).float().cpu().numpy()
        np.testing.assert_allclose(Y, c["Y"], rtol=tol, atol=tol)


@pytest.mark.parametrize("k", [1, 3, 7, 16, 64, 72])
@pytest.mark.parametrize("it", [np.int32, np.int64])
def test_parity_fp32(ms, orc, k, it):
    (d, i, p), shape = wl.ragged_csr(1500, 900, 3, 20, it)
    B = wl.uniform_matrix(shape[1], k, 4)
    Y = (_csr(ms, d, i, p, shape) @ _dev(B)).cpu().numpy()
    Y_ref = orc.csr_matmul(d, i, p, B, shape[0], workers=8)
    np.testing.assert_allclose(Y, Y_ref, rtol=1e-5, atol=1e-5)
    np.testing.assert_array_equal(Y, Y_ref)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_half_types(ms, orc, dtype):
    (d, i, p), shape = wl.random_k_per_row(2000, 1500, 16, 8)
    B = wl.uniform_matrix(shape[1], 64, 9)
    Y = (_csr(ms, d, i, p, shape, dtype) @ _dev(B).to(dtype)).float().cpu().numpy()
    if dtype == torch.float16:
        Y_ref = orc.csr_matmul(d.astype(np.float16), i, p, B.astype(np.float16), shape[0]).astype(np.float32)
        tol = 5e-3
    else:
        Y_ref = orc.bf16_bits_to_f32(orc.csr_matmul(orc.f32_to_bf16_bits(d), i, p, orc.f32_to_bf16_bits(B),
                                                    shape[0], bf16=True))
        tol = 1e-2
    np.testing.assert_allclose(Y, Y_ref, rtol=tol, atol=tol)


def test_column_slabs_larger_than_l2_budget(ms, orc):
    # n_cols * k * 4 B = 64 MiB > half the L2: the RHS is processed in >= 2 slabs
    (d, i, p), shape = wl.random_k_per_row(4096, 1 << 18, 16, 10)
    B = wl.uniform_matrix(shape[1], 64, 11)
    Y = (_csr(ms, d, i, p, shape) @ _dev(B)).cpu().numpy()
    Y_ref = orc.csr_matmul(d, i, p, B, shape[0], workers=8)
    np.testing.assert_array_equal(Y, Y_ref)


def test_batched_rhs(ms, orc):
    (d, i, p), shape = wl.ragged_csr(300, 200, 5, 10)
    B = np.stack([wl.uniform_matrix(shape[1], 8, s) for s in range(3)])
    Y = (_csr(ms, d, i, p, shape) @ _dev(B)).cpu().numpy()
    for s in range(3):
        np.testing.assert_allclose(Y[s], orc.csr_matmul(d, i, p, B[s], shape[0]), rtol=1e-5, atol=1e-5)


def test_empty_rows_and_zero_width(ms):
    A = ms.csr_array((torch.tensor([1.0, 2.0], device="cuda"), torch.tensor([0, 1], dtype=torch.int32,
                                                                            device="cuda"),
                      torch.tensor([0, 0, 2, 2], dtype=torch.int32, device="cuda")), shape=(3, 2))
    Y = A @ torch.ones((2, 4), device="cuda")
    assert Y.cpu().tolist() == [[0.0] * 4, [3.0] * 4, [0.0] * 4]
    assert (A @ torch.ones((2, 0), device="cuda")).shape == (3, 0)


@pytest.mark.parametrize("bf16", [False, True], ids=["f32", "bf16"])
def test_full_size_baseline_config(ms, orc, bf16):
    """BASELINE config 2 at full size: 2^20 x 2^20, 16 nonzeros per row, k = 64
    (seeds as bench.py). fp32 bit-exact; bf16 (fp32 accumulation, one rounding
    at the store) within 1e-2 relative per element of max(|Y|, sum |a b|)."""
    n, k = 1 << 20, 64
    (d, i, p), shape = wl.random_k_per_row(n, n, 16, 2)
    B = np.random.default_rng(102).uniform(-1, 1, (n, k)).astype(np.float32)
    if not bf16:
        Y = (_csr(ms, d, i, p, shape) @ _dev(B)).cpu().numpy()
        Y_ref = orc.csr_matmul(d, i, p, B, n, workers=8)
        np.testing.assert_array_equal(Y, Y_ref)
        return
    A = _csr(ms, d, i, p, shape, torch.bfloat16)
    Y = (A @ _dev(B).to(torch.bfloat16)).float().cpu().numpy()
    db, Bb = orc.f32_to_bf16_bits(d), orc.f32_to_bf16_bits(B)
    Y_ref = orc.bf16_bits_to_f32(orc.csr_matmul(db, i, p, Bb, n, bf16=True, workers=8))
    scale = orc.csr_matmul(np.abs(orc.bf16_bits_to_f32(db)), i, p, np.abs(orc.bf16_bits_to_f32(Bb)), n, workers=8)
    err = np.abs(Y.astype(np.float64) - Y_ref)
    assert np.all(err <= 1e-2 * np.maximum(np.abs(Y_ref), scale)), float(np.max(err / np.maximum(scale, 1e-30)))


@pytest.mark.parametrize("chunks", [1, 3, 8])
def test_streamed_host_operands_equal_the_device_product(ms, chunks):
    """csr_matmul_streamed (host operands, pipelined uploads / row-block
    products / downloads) gives the device product bit for bit, also with
    empty rows and blocks without nonzeros."""
    (d, i, p), shape = wl.ragged_csr(5000, 3000, 6, 40)
    B = wl.uniform_matrix(shape[1], 48, 7)
    A_host = ms.CSRArray(torch.from_numpy(d).pin_memory(), torch.from_numpy(i).pin_memory(),
                         torch.from_numpy(p).pin_memory(), shape, has_canonical_format=True)
    Y = ms.csr_matmul_streamed(A_host, torch.from_numpy(B).pin_memory(), chunks=chunks)
    assert not Y.is_cuda
    Y_dev = (_csr(ms, d, i, p, shape) @ _dev(B)).cpu()
    assert torch.equal(Y, Y_dev)
    out = torch.empty_like(Y).pin_memory()
    ms.csr_matmul_streamed(A_host, torch.from_numpy(B), chunks=chunks, out=out)
    assert torch.equal(out, Y_dev)
