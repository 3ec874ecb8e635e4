"""Metadata validation with the reference's messages.

Restates mlx-sparse's ``mlx_sparse/_validation.py`` checks on the product path
(``check_rank1``/``check_index_dtype``/``check_value_dtype`` :78-93,
``validate_csr_metadata`` :96-125, ``validate_csr_matvec_inputs`` :251-265,
``validate_csr_matmul_inputs`` :324-339): ranks, lengths and dtypes only, never
the array values, so validation needs no device synchronisation.
"""

from __future__ import annotations

import numpy as np
import torch

VALUE_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
INDEX_DTYPES = (torch.int32, torch.int64)

_NUMPY_TO_TORCH = {
    np.dtype(np.float32): torch.float32,
    np.dtype(np.float16): torch.float16,
    np.dtype(np.float64): torch.float32,
    np.dtype(np.int32): torch.int32,
    np.dtype(np.int64): torch.int64,
}


def _dtype_name(dt) -> str:
    return str(dt).split(".")[-1]


def default_device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("mlx_sparse (B200 build) needs a CUDA device; none is available.")
    return torch.device("cuda", torch.cuda.current_device())


def ensure_array(value, *, dtype=None, device=None) -> torch.Tensor:
    """Converts array-likes to a CUDA tensor (the role of ``ensure_mx_array``)."""
    if isinstance(value, torch.Tensor):
        t = value
        if dtype is not None and t.dtype != dtype:
            t = t.to(dtype)
        if not t.is_cuda:
            t = t.to(device or default_device())
        return t
    arr = np.asarray(value)
    tdt = dtype if dtype is not None else _NUMPY_TO_TORCH.get(arr.dtype)
    if tdt is None:
        if arr.dtype.kind == "f":
            tdt = torch.float32
        elif arr.dtype.kind in "iu":
            tdt = torch.int64
        else:
            raise TypeError(f"unsupported array dtype {arr.dtype}.")
    return torch.as_tensor(np.ascontiguousarray(arr)).to(device=device or default_device(), dtype=tdt)


def check_rank1(name: str, array) -> None:
    if array.ndim != 1:
        raise ValueError(f"{name} must be rank-1, got shape={tuple(array.shape)}.")


def check_index_dtype(name: str, array) -> None:
    if array.dtype not in INDEX_DTYPES:
        allowed = ", ".join(_dtype_name(dt) for dt in INDEX_DTYPES)
        raise TypeError(f"{name} dtype must be one of {allowed}, got {_dtype_name(array.dtype)}.")


def check_value_dtype(name: str, array) -> None:
    if array.dtype not in VALUE_DTYPES:
        allowed = ", ".join(_dtype_name(dt) for dt in VALUE_DTYPES)
        raise TypeError(f"{name} dtype must be one of {allowed}, got {_dtype_name(array.dtype)}.")


def normalize_shape(shape) -> tuple[int, int]:
    try:
        n_rows, n_cols = (int(s) for s in shape)
    except Exception as exc:
        raise ValueError(f"shape must be a length-2 sequence, got {shape!r}.") from exc
    if n_rows < 0 or n_cols < 0:
        raise ValueError(f"shape dimensions must be non-negative, got {(n_rows, n_cols)}.")
    return n_rows, n_cols


def validate_csr_metadata(data, indices, indptr, shape) -> None:
    check_rank1("CSRArray.data", data)
    check_rank1("CSRArray.indices", indices)
    check_rank1("CSRArray.indptr", indptr)
    check_value_dtype("CSRArray.data", data)
    check_index_dtype("CSRArray.indices", indices)
    check_index_dtype("CSRArray.indptr", indptr)
    if indices.dtype != indptr.dtype:
        raise TypeError(
            "CSRArray indices and indptr must have the same dtype, "
            f"got {_dtype_name(indices.dtype)} and {_dtype_name(indptr.dtype)}."
        )
    if data.shape[0] != indices.shape[0]:
        raise ValueError(
            "CSRArray data and indices must have the same length, "
            f"got {data.shape[0]} and {indices.shape[0]}."
        )
    if indptr.shape[0] != shape[0] + 1:
        raise ValueError(
            "CSRArray indptr must have shape (n_rows + 1,), "
            f"got {tuple(indptr.shape)} for n_rows={shape[0]}."
        )


def validate_csr_values(indices, indptr, shape, nnz: int) -> None:
    """``validate="full"``: indptr monotone, endpoints, column bounds (syncs)."""
    ip = indptr.detach().to("cpu").numpy()
    if ip.shape[0] and (int(ip[0]) != 0 or int(ip[-1]) != nnz):
        raise ValueError(f"CSRArray indptr must start at 0 and end at nnz={nnz}.")
    if ip.shape[0] > 1 and np.any(np.diff(ip) < 0):
        raise ValueError("CSRArray indptr must be monotonically nondecreasing.")
    if nnz:
        lo, hi = int(indices.min().item()), int(indices.max().item())
        if lo < 0 or hi >= shape[1]:
            raise ValueError(
                f"CSRArray indices must be in bounds for n_cols={shape[1]}, got min={lo}, max={hi}."
            )


def validate_csr_matvec_inputs(data, indices, indptr, x, shape) -> None:
    validate_csr_metadata(data, indices, indptr, shape)
    if x.ndim != 1:
        raise ValueError(f"csr_matvec expects a rank-1 RHS, got shape={tuple(x.shape)}.")
    if x.shape[0] != shape[1]:
        raise ValueError(f"csr_matvec RHS has length {x.shape[0]}, but sparse n_cols={shape[1]}.")
    check_value_dtype("csr_matvec data", data)
    check_value_dtype("csr_matvec RHS", x)
    if data.dtype != x.dtype:
        raise TypeError(
            "csr_matvec requires sparse data and RHS to have the same dtype, "
            f"got {_dtype_name(data.dtype)} and {_dtype_name(x.dtype)}."
        )


def validate_csr_matmul_inputs(data, indices, indptr, rhs, shape) -> None:
    validate_csr_metadata(data, indices, indptr, shape)
    if rhs.ndim != 2:
        raise ValueError(f"csr_matmul expects a rank-2 RHS, got shape={tuple(rhs.shape)}.")
    if rhs.shape[0] != shape[1]:
        raise ValueError(
            f"csr_matmul RHS has leading dimension {rhs.shape[0]}, but sparse n_cols={shape[1]}."
        )
    check_value_dtype("csr_matmul data", data)
    check_value_dtype("csr_matmul RHS", rhs)
    if data.dtype != rhs.dtype:
        raise TypeError(
            "csr_matmul requires sparse data and RHS to have the same dtype, "
            f"got {_dtype_name(data.dtype)} and {_dtype_name(rhs.dtype)}."
        )
