"""GPU test of msx_csr_matvec_noalloc, the SpMV entry point that allocates no
device memory (for callers that cannot allocate at call time: a pre-reserved
memory budget, or an execution phase where allocation is not allowed).

It is called through the C ABI and compared with the allocating stateless
entry point msx_csr_matvec(plan=NULL), on two calls in a row (the fixed
scratch array keeps the previous call's contents, which must not leak into
the next result). This file is collected last on purpose.
"""

import ctypes
import ctypes.util

import numpy as np
import pytest
import torch

import workloads as wl

pytestmark = pytest.mark.gpu


def _lib():
    from mlx_sparse import _native

    L = _native.extension()
    p, i64, c_int = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    L.msx_csr_matvec_noalloc.argtypes = [c_int, c_int, p, p, p, i64, p, p, i64, i64, p]
    return L, _native


_USED_MEM_CURRENT, _USED_MEM_HIGH = 7, 8  # cudaMemPoolAttrUsedMemCurrent / UsedMemHigh


def _cudart():
    for name in ("libcudart.so.12", "libcudart.so", ctypes.util.find_library("cudart")):
        if not name:
            continue
        try:
            return ctypes.CDLL(name)
        except OSError:
            continue
    pytest.skip("libcudart not loadable for the memory-pool check")


class _PoolWatch:
    """Peak of the device's default stream-ordered memory pool (the pool
    cudaMallocAsync draws from) across a region."""

    def __init__(self):
        self.rt = _cudart()
        self.pool = ctypes.c_void_p()
        assert self.rt.cudaDeviceGetDefaultMemPool(ctypes.byref(self.pool), torch.cuda.current_device()) == 0

    def _get(self, attr):
        v = ctypes.c_uint64()
        assert self.rt.cudaMemPoolGetAttribute(self.pool, attr, ctypes.byref(v)) == 0
        return v.value

    def __enter__(self):
        torch.cuda.synchronize()
        zero = ctypes.c_uint64(0)
        assert self.rt.cudaMemPoolSetAttribute(self.pool, _USED_MEM_HIGH, ctypes.byref(zero)) == 0
        self.before = self._get(_USED_MEM_CURRENT)
        self.torch_before = torch.cuda.memory_stats().get("allocation.all.allocated", 0)
        return self

    def __exit__(self, *exc):
        torch.cuda.synchronize()
        self.peak_growth = self._get(_USED_MEM_HIGH) - self.before
        self.torch_allocs = torch.cuda.memory_stats().get("allocation.all.allocated", 0) - self.torch_before


def _call(L, fn, A, x, y, stream, *plan):
    return fn(0, 0 if A[1].dtype == torch.int32 else 1, A[0].data_ptr(), A[1].data_ptr(), A[2].data_ptr(),
              A[0].numel(), x.data_ptr(), y.data_ptr(), A[2].numel() - 1, x.numel(), *plan, stream)


@pytest.mark.parametrize("make", [lambda: wl.ragged_csr(4000, 3000, 7, 40),   # rows split across tiles
                                  lambda: wl.lap2d(200, np.int64)], ids=["ragged", "lap2d_i64"])
def test_noalloc_matches_allocating_entry_point(make):
    L, native = _lib()
    (d, i, p), shape = make()
    A = tuple(torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (d, i, p))
    stream = torch.cuda.current_stream().cuda_stream
    for seed in (1, 2):  # two calls in a row, different inputs
        x = torch.from_numpy(wl.uniform_vector(shape[1], seed)).cuda()
        y_ref = torch.empty(shape[0], device="cuda")
        native.check(_call(L, L.msx_csr_matvec, A, x, y_ref, stream, None))
        y = torch.full((shape[0],), float("nan"), device="cuda")
        with _PoolWatch() as w:
            native.check(_call(L, L.msx_csr_matvec_noalloc, A, x, y, stream))
        assert w.peak_growth == 0 and w.torch_allocs == 0, (w.peak_growth, w.torch_allocs)
        torch.cuda.synchronize()
        np.testing.assert_allclose(y.cpu().numpy(), y_ref.cpu().numpy(), rtol=1e-5, atol=1e-5)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    L, _ = _lib()
    buf = torch.zeros(16, device="cuda")
    rc = L.msx_csr_matvec_noalloc(0, 0, buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), 1 << 40, buf.data_ptr(),
                                  buf.data_ptr(), 1 << 20, 1 << 20, None)
    assert rc == 1
    assert b"scratch" in L.msx_last_error()


def test_pool_watch_sees_the_allocating_entry_point():
    """The allocation check above is meaningful: the stateless entry point's
    stream-ordered scratch shows up in the same pool statistics."""
    L, native = _lib()
    (d, i, p), shape = wl.ragged_csr(4000, 3000, 7, 40)
    A = tuple(torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (d, i, p))
    x = torch.from_numpy(wl.uniform_vector(shape[1], 3)).cuda()
    y = torch.empty(shape[0], device="cuda")
    with _PoolWatch() as w:
        native.check(_call(L, L.msx_csr_matvec, A, x, y, torch.cuda.current_stream().cuda_stream, None))
    assert w.peak_growth > 0
