"""Public product ops: ``csr_matvec``, ``csr_matmul``, ``csr_matmat``.

Mirror mlx-sparse's ``mlx_sparse/_ops.py`` (``csr_matvec`` :780-818,
``csr_matmat`` :855-910, ``csr_matmul`` :1118-1167): type checks, metadata
validation, then the native call. Results are enqueued on the current CUDA
stream; only ``csr_matmat`` synchronises (its output size is data dependent,
as in the reference's host path).
"""

from __future__ import annotations

from mlx_sparse import _native
from mlx_sparse._csr import CSRArray
from mlx_sparse._validation import (
    ensure_array,
    validate_csr_matmul_inputs,
    validate_csr_matvec_inputs,
)


def csr_matvec(a: CSRArray, x):
    """``y = A @ x`` for a rank-1 dense ``x`` (same dtype as ``a.data``)."""
    if not isinstance(a, CSRArray):
        raise TypeError(f"csr_matvec expects CSRArray, got {type(a).__name__}.")
    x = ensure_array(x, device=a.device)
    validate_csr_matvec_inputs(a.data, a.indices, a.indptr, x, a.shape)
    plan = a.spmv_plan() if a.shape[0] > 0 else None
    return _native.csr_matvec(a.data, a.indices, a.indptr, x, a.shape, plan=plan)


def csr_matmul(a: CSRArray, rhs):
    """``Y = A @ B`` for a rank-2 dense ``B``; rank >= 3 is a batch of matrices
    (``rhs.shape[-2]`` is the sparse dimension), one native batched call."""
    if not isinstance(a, CSRArray):
        raise TypeError(f"csr_matmul expects CSRArray, got {type(a).__name__}.")
    rhs = ensure_array(rhs, device=a.device)
    if rhs.ndim == 2:
        validate_csr_matmul_inputs(a.data, a.indices, a.indptr, rhs, a.shape)
        return _native.csr_matmul(a.data, a.indices, a.indptr, rhs, a.shape)
    if rhs.ndim < 2:
        raise ValueError(f"csr_matmul expects rank-2 or higher RHS, got {tuple(rhs.shape)}.")
    if rhs.shape[-2] != a.shape[1]:
        raise ValueError(
            f"csr_matmul RHS has sparse dimension {rhs.shape[-2]}, but sparse n_cols={a.shape[1]}."
        )
    return _csr_matmul_batched(a, rhs)


def _csr_matmul_batched(a: CSRArray, rhs):
    """Reference: ``_ops._csr_matmul_batched`` (``mlx_sparse/_ops.py:985-998``)."""
    if a.data.dtype != rhs.dtype:
        raise TypeError(
            "csr_matmul requires sparse data and RHS to have the same dtype, "
            f"got {a.data.dtype} and {rhs.dtype}."
        )
    batch_shape = tuple(int(d) for d in rhs.shape[:-2])
    k = int(rhs.shape[-1])
    flat = rhs.reshape(-1, a.shape[1], k)
    out = _native.csr_batched_matmul(a.data, a.indices, a.indptr, flat, a.shape)
    return out.reshape(*batch_shape, a.shape[0], k)


def csr_batched_matmul(a: CSRArray, rhs):
    """``Y[..] = A @ B[..]`` for ``rhs`` of shape ``(..., n_cols, k)``, rank >= 3.

    Reference: ``_ops.csr_batched_matmul`` (``mlx_sparse/_ops.py:1097-1115``).
    """
    if not isinstance(a, CSRArray):
        raise TypeError(f"csr_batched_matmul expects CSRArray, got {type(a).__name__}.")
    rhs = ensure_array(rhs, device=a.device)
    if rhs.ndim < 3:
        raise ValueError(f"csr_batched_matmul expects rank-3 or higher RHS, got {tuple(rhs.shape)}.")
    if rhs.shape[-2] != a.shape[1]:
        raise ValueError(
            f"csr_batched_matmul RHS has sparse dimension {rhs.shape[-2]}, but sparse n_cols={a.shape[1]}."
        )
    return _csr_matmul_batched(a, rhs)


def csr_batched_matvec(a: CSRArray, rhs):
    """``Y[..] = A @ X[..]`` for ``rhs`` of shape ``(..., n_cols)``, rank >= 2.

    Reference: ``_ops.csr_batched_matvec`` (``mlx_sparse/_ops.py:821-852``).
    """
    if not isinstance(a, CSRArray):
        raise TypeError(f"csr_batched_matvec expects CSRArray, got {type(a).__name__}.")
    rhs = ensure_array(rhs, device=a.device)
    if rhs.ndim < 2:
        raise ValueError(f"csr_batched_matvec expects rank-2 or higher RHS, got {tuple(rhs.shape)}.")
    if rhs.shape[-1] != a.shape[1]:
        raise ValueError(
            f"csr_batched_matvec RHS has vector dimension {rhs.shape[-1]}, but sparse n_cols={a.shape[1]}."
        )
    if a.data.dtype != rhs.dtype:
        raise TypeError(
            "csr_batched_matvec requires sparse data and RHS to have the same dtype, "
            f"got {a.data.dtype} and {rhs.dtype}."
        )
    batch_shape = tuple(int(d) for d in rhs.shape[:-1])
    flat = rhs.reshape(-1, a.shape[1])
    out = _native.csr_batched_matvec(a.data, a.indices, a.indptr, flat, a.shape)
    return out.reshape(*batch_shape, a.shape[0])


def csr_matmat(a: CSRArray, rhs: CSRArray) -> CSRArray:
    """``C = A @ B`` for two CSR matrices; returns canonical CSR."""
    if not isinstance(a, CSRArray):
        raise TypeError(f"csr_matmat expects CSRArray lhs, got {type(a).__name__}.")
    if not isinstance(rhs, CSRArray):
        raise TypeError(f"csr_matmat expects CSRArray rhs, got {type(rhs).__name__}.")
    if a.data.dtype != rhs.data.dtype:
        raise TypeError(
            "CSR sparse-sparse matmul requires matching value dtypes, "
            f"got {a.data.dtype} and {rhs.data.dtype}."
        )
    if a.shape[1] != rhs.shape[0]:
        raise ValueError("CSR sparse-sparse matmul dimension mismatch.")
    data, indices, indptr = _native.csr_matmat(a, rhs)
    return CSRArray(data, indices, indptr, (a.shape[0], rhs.shape[1]), sorted_indices=True,
                    has_canonical_format=True)
