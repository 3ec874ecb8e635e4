"""``COOArray``: coordinate-format entry into the product path.

Mirrors the parts of mlx-sparse's ``mlx_sparse/_coo.py`` that feed the path:
the container, ``tocsr`` (:126-154: rows sorted, duplicates kept unless
``canonical=True``) and ``__matmul__`` (:245-268, which multiplies through CSR).
"""

from __future__ import annotations

from dataclasses import dataclass

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

    def __post_init__(self) -> None:
        object.__setattr__(self, "shape", normalize_shape(self.shape))

    @property
    def nnz(self) -> int:
        return int(self.data.shape[0])

    @property
    def dtype(self):
        return self.data.dtype

    def tocsr(self, *, canonical: bool = False) -> CSRArray:
        """Rows sorted (stable, so entries keep their order within a row)."""
        n_rows = self.shape[0]
        row = self.row.to(torch.int64)
        order = torch.sort(row, stable=True).indices
        counts = torch.bincount(row, minlength=n_rows)
        indptr = torch.zeros(n_rows + 1, dtype=torch.int64, device=self.data.device)
        torch.cumsum(counts, 0, out=indptr[1:])
        it = self.col.dtype
        csr = CSRArray(self.data[order].contiguous(), self.col[order].to(it).contiguous(), indptr.to(it),
                       self.shape, sorted_indices=False, has_canonical_format=False)
        return csr.canonicalize() if canonical else csr

    def __matmul__(self, rhs):
        return self.tocsr(canonical=True) @ rhs


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
