"""TEST INFRASTRUCTURE ONLY - numpy/ctypes front-end of the CPU oracle.

Wraps ``liboracle.so`` (``oracle.cpp``: a C++ restatement of mlx-sparse's CPU
loops for SpMV, SpMM, SpGEMM, CG and Jacobi-PCG, each function citing the
reference lines it follows). Used by ``tests/`` as the parity checker and by
``bench.py`` as the timed CPU baseline; the product path never imports it.

Parity is pinned by ``tests/test_oracle.py``: the oracle reproduces every
known-answer case of the reference's own tests for this path
(tests/test_csr_matvec.py:25-36, tests/test_csr_matmul.py:25-45,383-432,480-517,
tests/test_linalg_preconditioners.py:1977-2123) and agrees with SciPy, the
secondary oracle those tests use.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_VT = {np.dtype(np.float32): 0, np.dtype(np.float16): 1}
_IT = {np.dtype(np.int32): 0, np.dtype(np.int64): 1}

# bf16 arrays are carried as uint16 bit patterns on the numpy side.
BF16 = "bf16"


def build() -> str:
    """Compiles liboracle.so if it is missing or older than oracle.cpp. Holds a
    file lock while it checks and builds, so processes that start together
    (multi-rank tests) build it once; the library is written under a
    temporary name and renamed into place."""
    import fcntl

    src = os.path.join(HERE, "oracle.cpp")
    with open(os.path.join(HERE, ".build.lock"), "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
            subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        c_i64, c_int, c_float, p = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_void_p
        L.orc_last_error.restype = ctypes.c_char_p
        L.orc_csr_matvec.argtypes = [c_int, c_int, p, p, p, p, p, c_i64, c_int]
        L.orc_csr_matmul.argtypes = [c_int, c_int, p, p, p, p, c_i64, p, c_i64, c_int]
        L.orc_csr_matmat.argtypes = [c_int, c_int, p, p, p, c_int, p, p, p, c_i64, c_i64, c_i64]
        L.orc_csr_matmat.restype = p
        L.orc_matmat_nnz.argtypes = [p]
        L.orc_matmat_nnz.restype = c_i64
        L.orc_matmat_copy.argtypes = [p, p, p, p]
        L.orc_matmat_free.argtypes = [p]
        L.orc_csr_cg.argtypes = [c_int, p, p, p, p, p, p, c_i64, c_float, c_float, c_int, p, p, p]
        L.orc_csr_pcg_jacobi.argtypes = [c_int, p, p, p, p, p, p, p, c_i64, c_float, c_float, c_int, p, p, p, c_int]
        L.orc_weighted_ranges.argtypes = [p, c_i64, c_int, p]
        L.orc_coo_tocsr.argtypes = [c_int, c_int, p, p, p, c_i64, c_i64, c_int, p, p, p, p]
        L.orc_coo_matmul.argtypes = [c_int, c_int, p, p, p, c_i64, p, c_i64, p, c_i64]
        L.orc_csr_matmul_transpose.argtypes = [c_int, c_int, p, p, p, c_i64, c_i64, p, c_i64, p]
        L.orc_csr_data_vjp.argtypes = [c_int, c_int, p, p, c_i64, p, p, c_i64, p]
        L.orc_chebyshev_apply.argtypes = [c_int, p, p, p, c_i64, p, c_i64, p, c_int, c_float, c_float]
        L.orc_csr_pcg_chebyshev.argtypes = [c_int, p, p, p, p, p, p, p, p, p, c_i64, c_int, c_float, c_float,
                                            c_float, c_float, c_int, p, p, p]
        L.orc_gershgorin.argtypes = [c_int, p, p, p, c_i64, p]
        _lib = L
    return _lib


def _ptr(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _vt(values: np.ndarray, bf16: bool) -> int:
    if bf16:
        assert values.dtype == np.uint16
        return 2
    return _VT[values.dtype]


def _check(rc: int):
    if rc != 0:
        raise RuntimeError(lib().orc_last_error().decode())


def default_workers() -> int:
    """The reference's auto worker count (src/common/cpu_parallel.cpp:97-123)."""
    for name in ("OMP_NUM_THREADS", "SLURM_CPUS_PER_TASK", "PBS_NP", "LSB_DJOB_NUMPROC", "NSLOTS"):
        try:
            v = int(os.environ.get(name, ""))
            if v > 0:
                return v
        except ValueError:
            pass
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def csr_matvec(data, indices, indptr, x, n_rows, *, bf16=False, workers=1):
    data, indices, indptr, x = (np.ascontiguousarray(a) for a in (data, indices, indptr, x))
    y = np.empty(n_rows, dtype=data.dtype)
    _check(lib().orc_csr_matvec(_vt(data, bf16), _IT[indices.dtype], _ptr(data), _ptr(indices), _ptr(indptr),
                                _ptr(x), _ptr(y), n_rows, workers))
    return y


def csr_matmul(data, indices, indptr, rhs, n_rows, *, bf16=False, workers=1):
    data, indices, indptr, rhs = (np.ascontiguousarray(a) for a in (data, indices, indptr, rhs))
    k = rhs.shape[1]
    out = np.empty((n_rows, k), dtype=data.dtype)
    _check(lib().orc_csr_matmul(_vt(data, bf16), _IT[indices.dtype], _ptr(data), _ptr(indices), _ptr(indptr),
                                _ptr(rhs), k, _ptr(out), n_rows, workers))
    return out


def csr_matmat(a, b, shape_a, shape_b, *, bf16=False):
    """a, b: (data, indices, indptr). Returns (data, indices, indptr) with the
    reference's output index dtype rule (csr_matmat.cpp:1354-1356)."""
    ad, ai, ap = (np.ascontiguousarray(v) for v in a)
    bd, bi, bp = (np.ascontiguousarray(v) for v in b)
    L = lib()
    h = L.orc_csr_matmat(_vt(ad, bf16), _IT[ai.dtype], _ptr(ad), _ptr(ai), _ptr(ap), _IT[bi.dtype], _ptr(bd),
                         _ptr(bi), _ptr(bp), shape_a[0], shape_b[0], shape_b[1])
    if not h:
        raise ValueError(L.orc_last_error().decode())
    try:
        nnz = L.orc_matmat_nnz(h)
        data = np.empty(nnz, dtype=ad.dtype)
        idx = np.empty(nnz, dtype=np.int64)
        ptr = np.empty(shape_a[0] + 1, dtype=np.int64)
        L.orc_matmat_copy(h, _ptr(data), _ptr(idx), _ptr(ptr))
    finally:
        L.orc_matmat_free(h)
    out_it = ai.dtype if ai.dtype == bi.dtype else np.dtype(np.int64)
    return data, idx.astype(out_it), ptr.astype(out_it)


def csr_cg(data, indices, indptr, b, x0, *, rtol, atol, maxiter):
    data, indices, indptr, b, x0 = (np.ascontiguousarray(a) for a in (data, indices, indptr, b, x0))
    n = b.shape[0]
    x = np.empty(n, dtype=np.float32)
    info, res, its = ctypes.c_int(), ctypes.c_float(), ctypes.c_int()
    _check(lib().orc_csr_cg(_IT[indices.dtype], _ptr(data), _ptr(indices), _ptr(indptr), _ptr(b), _ptr(x0),
                            _ptr(x), n, rtol, atol, maxiter, ctypes.byref(info), ctypes.byref(res),
                            ctypes.byref(its)))
    return x, info.value, res.value, its.value


def csr_pcg_jacobi(data, indices, indptr, b, x0, inv_diag, *, rtol, atol, maxiter, stop_after=0):
    data, indices, indptr, b, x0, inv_diag = (
        np.ascontiguousarray(a) for a in (data, indices, indptr, b, x0, inv_diag))
    n = b.shape[0]
    x = np.empty(n, dtype=np.float32)
    info, res, its = ctypes.c_int(), ctypes.c_float(), ctypes.c_int()
    _check(lib().orc_csr_pcg_jacobi(_IT[indices.dtype], _ptr(data), _ptr(indices), _ptr(indptr), _ptr(b),
                                    _ptr(x0), _ptr(inv_diag), _ptr(x), n, rtol, atol, maxiter, ctypes.byref(info),
                                    ctypes.byref(res), ctypes.byref(its), stop_after))
    return x, info.value, res.value, its.value


def coo_tocsr(data, row, col, n_rows, *, sort_columns=True, bf16=False):
    """(data, indices, indptr, perm): coo_tocsr.cpp:94-237 (sort_columns) or
    rows in source order (the coo_matmul summation order)."""
    data, row, col = (np.ascontiguousarray(a) for a in (data, row, col))
    nnz = row.shape[0]
    od = np.empty(nnz, dtype=data.dtype)
    oi = np.empty(nnz, dtype=col.dtype)
    op = np.empty(n_rows + 1, dtype=row.dtype)
    perm = np.empty(nnz, dtype=np.int64)
    _check(lib().orc_coo_tocsr(_vt(data, bf16), _IT[row.dtype], _ptr(data), _ptr(row), _ptr(col), nnz, n_rows,
                               int(sort_columns), _ptr(od), _ptr(oi), _ptr(op), _ptr(perm)))
    return od, oi, op, perm


def coo_matmul(data, row, col, rhs, n_rows, *, bf16=False):
    """coo_matmul.cpp: rows accumulated over entries in source order; rhs is
    (n_cols,) or (n_cols, k)."""
    data, row, col, rhs = (np.ascontiguousarray(a) for a in (data, row, col, rhs))
    k = 1 if rhs.ndim == 1 else rhs.shape[1]
    out = np.empty((n_rows, k), dtype=data.dtype)
    _check(lib().orc_coo_matmul(_vt(data, bf16), _IT[row.dtype], _ptr(data), _ptr(row), _ptr(col), row.shape[0],
                                _ptr(rhs), k, _ptr(out), n_rows))
    return out.reshape(n_rows) if rhs.ndim == 1 else out


def csr_matmul_transpose(data, indices, indptr, rhs, n_cols, *, bf16=False):
    """A^T @ rhs (csr_matvec_transpose.cpp:76-97 serial order); rhs (n_rows,)
    or (n_rows, k)."""
    data, indices, indptr, rhs = (np.ascontiguousarray(a) for a in (data, indices, indptr, rhs))
    n_rows = indptr.shape[0] - 1
    k = 1 if rhs.ndim == 1 else rhs.shape[1]
    out = np.empty((n_cols, k), dtype=data.dtype)
    _check(lib().orc_csr_matmul_transpose(_vt(data, bf16), _IT[indices.dtype], _ptr(data), _ptr(indices),
                                          _ptr(indptr), n_rows, n_cols, _ptr(rhs), k, _ptr(out)))
    return out.reshape(n_cols) if rhs.ndim == 1 else out


def csr_data_vjp(indices, indptr, rhs, cot, *, bf16=False):
    """csr_matvec_data_vjp (rhs, cot rank 1) / csr_matmul_data_vjp (rank 2)."""
    indices, indptr, rhs, cot = (np.ascontiguousarray(a) for a in (indices, indptr, rhs, cot))
    n_rows = indptr.shape[0] - 1
    k = 1 if rhs.ndim == 1 else rhs.shape[1]
    out = np.empty(indices.shape[0], dtype=rhs.dtype)
    _check(lib().orc_csr_data_vjp(_vt(rhs, bf16), _IT[indices.dtype], _ptr(indices), _ptr(indptr), n_rows,
                                  _ptr(rhs), _ptr(cot), k, _ptr(out)))
    return out


def chebyshev_apply(data, indices, indptr, rhs, *, degree, lambda_min, lambda_max):
    data, indices, indptr, rhs = (np.ascontiguousarray(a) for a in (data, indices, indptr, rhs))
    n = indptr.shape[0] - 1
    k = 1 if rhs.ndim == 1 else rhs.shape[1]
    out = np.empty((n, k), dtype=np.float32)
    _check(lib().orc_chebyshev_apply(_IT[indices.dtype], _ptr(data), _ptr(indices), _ptr(indptr), n, _ptr(rhs), k,
                                     _ptr(out), int(degree), float(lambda_min), float(lambda_max)))
    return out.reshape(n) if rhs.ndim == 1 else out


def csr_pcg_chebyshev(data, indices, indptr, b, x0, m, *, degree, lambda_min, lambda_max, rtol, atol, maxiter):
    """m = (data, indices, indptr) of the preconditioner matrix."""
    data, indices, indptr, b, x0 = (np.ascontiguousarray(a) for a in (data, indices, indptr, b, x0))
    md, mi, mp = (np.ascontiguousarray(a) for a in m)
    n = b.shape[0]
    x = np.empty(n, dtype=np.float32)
    info, res, its = ctypes.c_int(), ctypes.c_float(), ctypes.c_int()
    _check(lib().orc_csr_pcg_chebyshev(_IT[indices.dtype], _ptr(data), _ptr(indices), _ptr(indptr), _ptr(b),
                                       _ptr(x0), _ptr(md), _ptr(mi), _ptr(mp), _ptr(x), n, int(degree),
                                       float(lambda_min), float(lambda_max), rtol, atol, maxiter,
                                       ctypes.byref(info), ctypes.byref(res), ctypes.byref(its)))
    return x, info.value, res.value, its.value


def gershgorin(data, indices, indptr):
    """(lower, upper, diag_min, diag_max) of chebyshev.cpp:120-161."""
    data, indices, indptr = (np.ascontiguousarray(a) for a in (data, indices, indptr))
    out = np.empty(4, dtype=np.float32)
    _check(lib().orc_gershgorin(_IT[indices.dtype], _ptr(data), _ptr(indices), _ptr(indptr), indptr.shape[0] - 1,
                                _ptr(out)))
    return tuple(float(v) for v in out)


REF_LIB = os.path.join(HERE, "_ref", "libref_parallel.so")


def build_ref() -> str | None:
    """Compiles oracle/_ref/libref_parallel.so from the reference's own
    src/common/cpu_parallel.cpp when the reference checkout is present
    (MSX_REFERENCE_ROOT, default: a `reference` folder beside the repository);
    returns its path or None."""
    root = os.environ.get("MSX_REFERENCE_ROOT", os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference"))
    if not os.path.exists(os.path.join(root, "src", "common", "cpu_parallel.cpp")):
        return REF_LIB if os.path.exists(REF_LIB) else None
    subprocess.run(["make", "-s", "-C", HERE, "ref", f"REF={root}"], check=True)
    return REF_LIB


def ref_weighted_ranges(work, parts):
    """The reference's weighted_cpu_ranges (cpu_parallel.cpp:202-253), run from
    its own source compiled by build_ref(); list of (begin, end)."""
    L = ctypes.CDLL(REF_LIB)
    L.ref_weighted_ranges.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
    w = np.ascontiguousarray(work, dtype=np.int64)
    out = np.empty(2 * max(parts, 1), dtype=np.int64)
    k = L.ref_weighted_ranges(_ptr(w), w.shape[0], parts, _ptr(out))
    return [(int(out[2 * i]), int(out[2 * i + 1])) for i in range(k)]


def weighted_ranges(work, parts):
    work = np.ascontiguousarray(work, dtype=np.int64)
    out = np.empty(2 * max(parts, 1), dtype=np.int64)
    n = lib().orc_weighted_ranges(_ptr(work), work.shape[0], parts, _ptr(out))
    return [(int(out[2 * i]), int(out[2 * i + 1])) for i in range(n)]


# ---- bf16 helpers (numpy has no bfloat16) -----------------------------------
def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (uint16)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(a, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)
