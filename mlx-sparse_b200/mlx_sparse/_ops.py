"""Public product ops: ``csr_matvec``, ``csr_matmul``, ``csr_matmat``.

Mirror mlx-sparse's ``mlx_sparse/_ops.py`` (``csr_matvec`` :780-818,
``csr_matmat`` :855-910, ``csr_matmul`` :1118-1167): type checks, metadata
validation, then the native call. Results are enqueued on the current CUDA
stream; only ``csr_matmat`` synchronises (its output size is data dependent,
as in the reference's host path).
"""

from __future__ import annotations

import torch

from mlx_sparse import _native
from mlx_sparse._coo import COOArray
from mlx_sparse._csr import CSRArray
from mlx_sparse._validation import (
    ensure_array,
    validate_csr_matmul_inputs,
    validate_csr_matvec_inputs,
)


def _wants_grad(*tensors) -> bool:
    return torch.is_grad_enabled() and any(t.requires_grad for t in tensors)


def csr_matvec(a: CSRArray, x):
    """``y = A @ x`` for a rank-1 dense ``x`` (same dtype as ``a.data``).

    Differentiable (torch autograd) in ``a.data`` and ``x``: the backward
    products are the reference's VJPs (``src/sparse/csr_matvec/
    csr_matvec.cpp:236-263``): ``csr_matvec_data_vjp`` and
    ``csr_matvec_transpose``.
    """
    if not isinstance(a, CSRArray):
        raise TypeError(f"csr_matvec expects CSRArray, got {type(a).__name__}.")
    x = ensure_array(x, device=a.device)
    validate_csr_matvec_inputs(a.data, a.indices, a.indptr, x, a.shape)
    if _wants_grad(a.data, x):
        from mlx_sparse._autodiff import CsrProduct

        return CsrProduct.apply(a.data, x, a)
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
        if _wants_grad(a.data, rhs):
            from mlx_sparse._autodiff import CsrProduct

            return CsrProduct.apply(a.data, rhs, a)
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


# ---------------------------------------------------------------------------
# Transposed products and data cotangents (the backward step of the products)
# ---------------------------------------------------------------------------
def csr_matvec_transpose(a: CSRArray, x):
    """``A^T @ x``. Reference: ``csr_matvec_transpose`` (``src/sparse/
    csr_matvec_transpose/csr_matvec_transpose.cpp:76-97``): each output entry
    sums its column's entries in row-major order. Runs as an SpMV over the
    matrix's cached transposed structure, which lists them in that order."""
    if not isinstance(a, CSRArray):
        raise TypeError(f"csr_matvec_transpose expects CSRArray, got {type(a).__name__}.")
    x = ensure_array(x, device=a.device)
    if x.ndim != 1 or x.shape[0] != a.shape[0]:
        raise ValueError(f"csr_matvec_transpose x must have shape ({a.shape[0]},), got {tuple(x.shape)}.")
    if x.dtype != a.data.dtype:
        raise TypeError(f"csr_matvec_transpose requires matching dtypes, got {a.data.dtype} and {x.dtype}.")
    return a.transpose() @ x


def csr_matmul_transpose(a: CSRArray, rhs):
    """``A^T @ B`` for ``B`` of shape ``(n_rows, k)`` (``src/sparse/
    csr_matmul_transpose``)."""
    if not isinstance(a, CSRArray):
        raise TypeError(f"csr_matmul_transpose expects CSRArray, got {type(a).__name__}.")
    rhs = ensure_array(rhs, device=a.device)
    if rhs.ndim != 2 or rhs.shape[0] != a.shape[0]:
        raise ValueError(f"csr_matmul_transpose rhs must have shape ({a.shape[0]}, k), got {tuple(rhs.shape)}.")
    if rhs.dtype != a.data.dtype:
        raise TypeError(f"csr_matmul_transpose requires matching dtypes, got {a.data.dtype} and {rhs.dtype}.")
    return a.transpose() @ rhs


def csr_matvec_data_vjp(a: CSRArray, x, cotangent):
    """Cotangent of ``a.data`` for ``y = A @ x``: ``cot[row(p)] * x[col(p)]``
    (``src/sparse/csr_matvec_data_vjp``)."""
    x = ensure_array(x, device=a.device)
    cotangent = ensure_array(cotangent, device=a.device)
    if x.shape != (a.shape[1],) or cotangent.shape != (a.shape[0],):
        raise ValueError("csr_matvec_data_vjp expects x of shape (n_cols,) and a cotangent of shape (n_rows,).")
    return _native.csr_data_vjp(a.indices, a.indptr, x, cotangent, a.shape)


def csr_matmul_data_vjp(a: CSRArray, rhs, cotangent):
    """Cotangent of ``a.data`` for ``Y = A @ B``: ``sum_j cot[row(p), j] *
    B[col(p), j]`` (``src/sparse/csr_matmul_data_vjp/
    csr_matmul_data_vjp.cpp:88-100``)."""
    rhs = ensure_array(rhs, device=a.device)
    cotangent = ensure_array(cotangent, device=a.device)
    if rhs.ndim != 2 or rhs.shape[0] != a.shape[1]:
        raise ValueError("csr_matmul_data_vjp rhs first dimension must equal the sparse matrix column count.")
    if cotangent.shape != (a.shape[0], rhs.shape[1]):
        raise ValueError("csr_matmul_data_vjp cotangent must have shape (n_rows, rhs_cols).")
    return _native.csr_data_vjp(a.indices, a.indptr, rhs, cotangent, a.shape)


# ---------------------------------------------------------------------------
# COO products
# ---------------------------------------------------------------------------
def _check_coo_rhs(a: COOArray, rhs, name):
    if rhs.dtype != a.data.dtype:
        raise TypeError(f"{name} requires sparse data and RHS to have the same dtype, got {a.data.dtype} and "
                        f"{rhs.dtype}.")


def coo_matvec(a: COOArray, x):
    """``y = A @ x`` for COO ``A``. Reference: ``coo_matvec`` (``src/sparse/
    coo_matmul/coo_matmul.cpp:343-357``), which sums every row over its
    entries in source order; the cached source-order CSR copy makes the same
    sums with the CSR SpMV kernels."""
    if not isinstance(a, COOArray):
        raise TypeError(f"coo_matvec expects COOArray, got {type(a).__name__}.")
    x = ensure_array(x, device=a.device)
    if x.ndim != 1 or x.shape[0] != a.shape[1]:
        raise ValueError(f"coo_matvec x must have shape ({a.shape[1]},), got {tuple(x.shape)}.")
    _check_coo_rhs(a, x, "coo_matvec")
    return csr_matvec(a._stored_order_csr(), x)


def coo_matmul(a: COOArray, rhs):
    """``Y = A @ B`` for COO ``A`` and a dense ``B`` (rank >= 2: batched).
    Reference: ``coo_matmul`` (``src/sparse/coo_matmul/coo_matmul.cpp:311-341``)."""
    if not isinstance(a, COOArray):
        raise TypeError(f"coo_matmul expects COOArray, got {type(a).__name__}.")
    rhs = ensure_array(rhs, device=a.device)
    if rhs.ndim < 2 or rhs.shape[-2] != a.shape[1]:
        raise ValueError("coo_matmul rhs first dimension must equal the sparse matrix column count.")
    _check_coo_rhs(a, rhs, "coo_matmul")
    return csr_matmul(a._stored_order_csr(), rhs)


def coo_matmat(a: COOArray, b: COOArray) -> COOArray:
    """Sparse-sparse product of COO operands; canonical COO result (as the
    reference's ``COOArray.__matmul__``), through the CSR SpGEMM kernels."""
    c = csr_matmat(a.tocsr(canonical=True), b.tocsr(canonical=True))
    return c.tocoo()


# ---------------------------------------------------------------------------
# Host-resident operands streamed through the GPU
# ---------------------------------------------------------------------------
def csr_matmul_streamed(a: CSRArray, rhs, *, device=None, chunks: int = 16, out=None):
    """``Y = A @ B`` for a CSR matrix and a dense ``B`` that live in host
    memory (pinned for full speed), computed on a GPU and returned in pinned
    host memory.

    The reference's arrays are host arrays (MLX unified memory); this entry
    keeps that calling convention while the product runs in the CUDA SpMM
    kernels. ``out`` may be a caller-owned pinned host tensor of shape
    ``(n_rows, k)`` (allocating pinned memory per call is slow). The
    transfers are pipelined on three streams: B and the row
    pointers go up first, then the matrix in ``chunks`` row blocks; each block
    is multiplied as soon as it has landed, and its rows of Y go back down
    while later blocks are still uploading (PCIe is full duplex). Nothing is
    computed on the CPU. Results equal ``A @ B`` on the device.
    """
    if not isinstance(a, CSRArray):
        raise TypeError(f"csr_matmul_streamed expects CSRArray, got {type(a).__name__}.")
    if not isinstance(rhs, torch.Tensor) or rhs.ndim != 2:
        raise ValueError("csr_matmul_streamed expects a rank-2 host tensor RHS.")
    if a.data.is_cuda or rhs.is_cuda:
        raise ValueError("csr_matmul_streamed takes host operands; use A @ B for device operands.")
    validate_csr_matmul_inputs(a.data, a.indices, a.indptr, rhs, a.shape)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    n_rows, n_cols = a.shape
    k = int(rhs.shape[1])
    if out is None:
        out = torch.empty((n_rows, k), dtype=a.data.dtype, pin_memory=True)
    elif out.is_cuda or tuple(out.shape) != (n_rows, k) or out.dtype != a.data.dtype or not out.is_contiguous():
        raise ValueError(f"csr_matmul_streamed out must be a contiguous host tensor of shape ({n_rows}, {k}).")
    if n_rows == 0 or k == 0:
        return out
    indptr_h = a.indptr.contiguous()
    ptr = indptr_h.numpy()  # only the block boundaries are read on the host
    with torch.cuda.device(dev):
        up, comp, down = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        cur = torch.cuda.current_stream(dev)
        up.wait_stream(cur)
        d_data = torch.empty(a.data.shape, dtype=a.data.dtype, device=dev)
        d_idx = torch.empty(a.indices.shape, dtype=a.indices.dtype, device=dev)
        d_out = torch.empty((n_rows, k), dtype=a.data.dtype, device=dev)
        with torch.cuda.stream(up):
            d_ptr = indptr_h.to(dev, non_blocking=True)
            d_rhs = rhs.contiguous().to(dev, non_blocking=True)
            ready_rhs = torch.cuda.Event()
            ready_rhs.record(up)
        bounds = [(n_rows * c) // chunks for c in range(chunks + 1)]
        for c in range(chunks):
            r0, r1 = bounds[c], bounds[c + 1]
            if r1 <= r0:
                continue
            k0, k1 = int(ptr[r0]), int(ptr[r1])
            with torch.cuda.stream(up):
                if k1 > k0:
                    d_data[k0:k1].copy_(a.data[k0:k1], non_blocking=True)
                    d_idx[k0:k1].copy_(a.indices[k0:k1], non_blocking=True)
                landed = torch.cuda.Event()
                landed.record(up)
            comp.wait_event(ready_rhs)
            comp.wait_event(landed)
            with torch.cuda.stream(comp):
                _native.csr_matmul(d_data, d_idx, d_ptr[r0:r1 + 1], d_rhs, (r1 - r0, n_cols), out=d_out[r0:r1])
                computed = torch.cuda.Event()
                computed.record(comp)
            down.wait_event(computed)
            with torch.cuda.stream(down):
                out[r0:r1].copy_(d_out[r0:r1], non_blocking=True)
        # the host waits for the last copy down (it waited on every block), so
        # the device buffers are free again when they are released
        down.synchronize()
    return out
