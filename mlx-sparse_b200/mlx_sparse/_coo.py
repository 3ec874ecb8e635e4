"""``COOArray``: coordinate-format entry into the product path.

Mirrors the parts of mlx-sparse's ``mlx_sparse/_coo.py`` that feed the path:
the container, ``tocsr`` (:126-154: entries sorted by row, then column, then
source position; duplicates kept unless ``canonical=True``) and ``__matmul__``
(:245-268: ``coo @ x`` / ``coo @ B`` through the native COO product, a sparse
right-hand side through the sparse-sparse product, returning COO).

Products with a dense right-hand side run on a cached CSR copy whose rows keep
the entries' source order, which is the summation order of the reference's
``coo_matmul`` (``src/sparse/coo_matmul/coo_matmul.cpp``), so the results are
the reference's bit for bit.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from mlx_sparse._csr import CSRArray
from mlx_sparse._validation import (
    check_index_dtype,
    check_rank1,
    check_value_dtype,
    ensure_array,
    normalize_shape,
)


@dataclass(frozen=True, slots=True)
class COOArray:
    data: torch.Tensor
    row: torch.Tensor
    col: torch.Tensor
    shape: tuple
    has_canonical_format: bool = False
    _cache: dict = field(default_factory=dict, repr=False, compare=False)

    def __post_init__(self) -> None:
        object.__setattr__(self, "shape", normalize_shape(self.shape))

    @property
    def nnz(self) -> int:
        return int(self.data.shape[0])

    @property
    def dtype(self):
        return self.data.dtype

    @property
    def index_dtype(self):
        return self.row.dtype

    @property
    def ndim(self) -> int:
        return 2

    @property
    def device(self):
        return self.data.device

    def tocsr(self, *, canonical: bool = False) -> CSRArray:
        """Converts on the device (``msx_coo_tocsr``): rows in order, each
        row by column then source position, duplicates kept; the result has
        ``sorted_indices=True``. ``canonical=True`` also sums duplicates."""
        from mlx_sparse import _native

        data, indices, indptr = _native.coo_tocsr(self.data, self.row, self.col, self.shape, sort_columns=True)
        csr = CSRArray(data, indices, indptr, self.shape, sorted_indices=True, has_canonical_format=False)
        return csr.canonicalize() if canonical else csr

    def _stored_order_csr(self) -> CSRArray:
        """CSR view whose rows keep the source order (products only). The
        structure and the permutation are cached; the values are gathered
        from ``self.data`` on each call, so autograd reaches ``self.data``."""
        if "csr" not in self._cache:
            from mlx_sparse import _native

            _, indices, indptr, perm = _native.coo_tocsr(self.data.detach(), self.row, self.col, self.shape,
                                                         sort_columns=False, with_perm=True)
            self._cache["csr"] = (indices, indptr, perm)
        indices, indptr, perm = self._cache["csr"]
        csr = CSRArray(self.data.index_select(0, perm), indices, indptr, self.shape)
        if "plan" in self._cache:
            csr._plan.append(self._cache["plan"])
        elif self.shape[0] > 0:
            self._cache["plan"] = csr.spmv_plan()
        return csr

    def todense(self) -> torch.Tensor:
        out = torch.zeros(self.shape, dtype=self.data.dtype, device=self.data.device)
        out.index_put_((self.row.to(torch.int64), self.col.to(torch.int64)), self.data, accumulate=True)
        return out

    def __matmul__(self, rhs):
        from mlx_sparse import _ops

        if isinstance(rhs, COOArray):
            return _ops.coo_matmat(self, rhs)
        if isinstance(rhs, CSRArray):
            return _ops.coo_matmat(self, rhs.tocoo())
        rhs = ensure_array(rhs, device=self.device)
        if rhs.ndim == 1:
            return _ops.coo_matvec(self, rhs)
        if rhs.ndim >= 2:
            return _ops.coo_matmul(self, rhs)
        raise ValueError(f"COO matmul expects rank-1 or higher RHS, got {tuple(rhs.shape)}.")


def coo_array(arg, shape, *, validate="metadata") -> COOArray:
    """Builds a ``COOArray`` from ``(data, (row, col))`` or ``(data, row, col)``."""
    shape = normalize_shape(shape)
    if isinstance(arg, COOArray):
        return arg
    try:
        if len(arg) == 2:
            data, (row, col) = arg
        else:
            data, row, col = arg
    except Exception as exc:
        raise TypeError("coo_array expects (data, (row, col)) or (data, row, col).") from exc
    data = ensure_array(data)
    row = ensure_array(row, device=data.device)
    col = ensure_array(col, device=data.device)
    if validate not in (False, "none"):
        check_rank1("COOArray.data", data)
        check_rank1("COOArray.row", row)
        check_rank1("COOArray.col", col)
        check_value_dtype("COOArray.data", data)
        check_index_dtype("COOArray.row", row)
        check_index_dtype("COOArray.col", col)
        if not (data.shape[0] == row.shape[0] == col.shape[0]):
            raise ValueError("COOArray data, row and col must have the same length.")
    return COOArray(data, row, col, shape)
