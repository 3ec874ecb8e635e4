"""``CSRArray``: the CSR container of the product path, on CUDA tensors.

Mirrors mlx-sparse's ``mlx_sparse/_csr.py`` (``CSRArray`` :33-120,
``canonicalize`` :239-250, ``__matmul__`` :502-552, ``csr_array`` :627-730): a
frozen dataclass of ``(data, indices, indptr, shape, sorted_indices,
has_canonical_format)`` whose ``@`` dispatches to SpMV, SpMM or SpGEMM by the
type and rank of the right-hand side. The arrays are torch CUDA tensors.

The B200 build adds one cache slot: the SpMV tile plan (nnz-balanced partition
of ``indptr``), built on the first product and reused while the instance lives.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch

from mlx_sparse import _native
from mlx_sparse._validation import (
    ensure_array,
    normalize_shape,
    validate_csr_metadata,
    validate_csr_values,
)


@dataclass(frozen=True, slots=True)
class CSRArray:
    """A 2D sparse matrix in Compressed Sparse Row format.

    Row ``i`` spans ``data[indptr[i]:indptr[i+1]]`` with column indices
    ``indices[indptr[i]:indptr[i+1]]``. ``data`` is float32, float16 or
    bfloat16; ``indices`` and ``indptr`` share int32 or int64. Duplicate
    columns are allowed unless ``has_canonical_format`` is set.
    """

    data: torch.Tensor
    indices: torch.Tensor
    indptr: torch.Tensor
    shape: tuple
    sorted_indices: bool = False
    has_canonical_format: bool = False
    _plan: list = field(default_factory=list, repr=False, compare=False)
    _solvers: dict = field(default_factory=dict, repr=False, compare=False)
    _cache: dict = field(default_factory=dict, repr=False, compare=False)

    def __post_init__(self) -> None:
        object.__setattr__(self, "shape", normalize_shape(self.shape))
        if self.has_canonical_format and not self.sorted_indices:
            object.__setattr__(self, "sorted_indices", True)

    @property
    def nnz(self) -> int:
        return int(self.data.shape[0])

    @property
    def dtype(self):
        return self.data.dtype

    @property
    def index_dtype(self):
        return self.indices.dtype

    @property
    def ndim(self) -> int:
        return 2

    @property
    def device(self):
        return self.data.device

    def spmv_plan(self) -> "_native.SpmvPlan":
        """The cached SpMV tile plan of this matrix (built on first use)."""
        if not self._plan:
            self._plan.append(_native.SpmvPlan(self.indptr.contiguous(), self.shape[0], self.nnz))
        return self._plan[0]

    def cg_context(self, preconditioned: bool) -> "_native.CgContext":
        """The cached persistent CG solver of this matrix (built on first use)."""
        key = bool(preconditioned)
        if key not in self._solvers:
            self._solvers[key] = _native.CgContext(self.data.contiguous(), self.indices.contiguous(),
                                                   self.indptr.contiguous(), self.shape[0], 0, key)
        return self._solvers[key]

    def canonicalize(self) -> "CSRArray":
        """Sorted indices, duplicates summed; ``self`` if already canonical."""
        if self.has_canonical_format:
            return self
        return self.sum_duplicates()

    def sum_duplicates(self) -> "CSRArray":
        """Sorts each row and sums entries sharing a column, in stored order.

        Runs as ``I @ self`` through the SpGEMM kernels with zero pruning off,
        so each output entry is the position-ordered sum of its duplicates.
        """
        n = self.shape[0]
        dev = self.data.device
        it = self.indices.dtype
        eye = CSRArray(
            data=torch.ones(n, dtype=self.data.dtype, device=dev),
            indices=torch.arange(n, dtype=it, device=dev),
            indptr=torch.arange(n + 1, dtype=it, device=dev),
            shape=(n, n),
            has_canonical_format=True,
        )
        data, indices, indptr = _native.csr_matmat(eye, self, prune_zeros=False)
        return CSRArray(data, indices, indptr, self.shape, sorted_indices=True, has_canonical_format=True)

    def transpose_structure(self):
        """``(indices, indptr, perm)`` of A^T (built once on the device by
        ``msx_csr_transpose`` and cached): row c of A^T lists column c's
        entries of A by ascending row, and ``perm`` maps them back to
        positions in ``data``."""
        if "t" not in self._cache:
            self._cache["t"] = _native.csr_transpose_structure(self.indices, self.indptr, self.shape)
        return self._cache["t"]

    def transpose(self) -> "CSRArray":
        """A^T as CSR (values gathered through the cached structure). Sorted
        indices; canonical when ``self`` is."""
        indices, indptr, perm = self.transpose_structure()
        data = self.data.detach().index_select(0, perm) if perm.numel() else self.data.detach()[:0]
        return CSRArray(data, indices, indptr, (self.shape[1], self.shape[0]), sorted_indices=True,
                        has_canonical_format=self.has_canonical_format)

    @property
    def T(self) -> "CSRArray":
        return self.transpose()

    def tocoo(self):
        """COO with the same entries in CSR order."""
        from mlx_sparse._coo import COOArray

        rows = torch.repeat_interleave(torch.arange(self.shape[0], device=self.device, dtype=self.indices.dtype),
                                       torch.diff(self.indptr.to(torch.int64)))
        return COOArray(self.data, rows, self.indices, self.shape, has_canonical_format=self.has_canonical_format)

    def diagonal(self) -> torch.Tensor:
        """Main diagonal as a dense vector (duplicate entries summed)."""
        return _native.csr_diagonal(self.data, self.indices, self.indptr, self.shape)

    def todense(self) -> torch.Tensor:
        rows = torch.repeat_interleave(
            torch.arange(self.shape[0], device=self.device), torch.diff(self.indptr.to(torch.int64))
        )
        out = torch.zeros(self.shape, dtype=self.data.dtype, device=self.device)
        out.index_put_((rows, self.indices.to(torch.int64)), self.data, accumulate=True)
        return out

    def astype(self, dtype) -> "CSRArray":
        return CSRArray(self.data.to(dtype), self.indices, self.indptr, self.shape, self.sorted_indices,
                        self.has_canonical_format)

    def __matmul__(self, rhs):
        """``A @ rhs``: SpGEMM for a sparse rhs, SpMV for a vector, SpMM for a matrix."""
        from mlx_sparse._coo import COOArray
        from mlx_sparse import _ops

        if isinstance(rhs, CSRArray):
            return _ops.csr_matmat(self, rhs)
        if isinstance(rhs, COOArray):
            return _ops.csr_matmat(self, rhs.tocsr(canonical=True))
        rhs = ensure_array(rhs, device=self.device)
        if rhs.ndim == 1:
            return _ops.csr_matvec(self, rhs)
        if rhs.ndim >= 2:
            return _ops.csr_matmul(self, rhs)
        raise ValueError(f"CSR matmul expects rank-1 or higher RHS, got {tuple(rhs.shape)}.")


def csr_array(arg, shape, *, validate="metadata", sorted_indices: bool = False, canonical=None) -> CSRArray:
    """Builds a ``CSRArray`` from ``(data, indices, indptr)`` or returns ``arg``.

    ``validate``: ``"metadata"`` (default; ranks/lengths/dtypes, no sync),
    ``"full"``/``True`` (also indptr monotonicity and column bounds; syncs), or
    ``False``/``"none"``.
    """
    mode = {True: "full", False: "none", None: "metadata"}.get(validate, validate)
    if mode not in ("metadata", "full", "none"):
        raise ValueError(f"validate must be 'metadata', 'full', 'none', True or False, got {validate!r}.")
    shape = normalize_shape(shape)
    if isinstance(arg, CSRArray):
        if arg.shape != shape:
            raise ValueError(f"CSRArray shape mismatch: got {arg.shape}, expected {shape}.")
        return arg
    try:
        data, indices, indptr = arg
    except Exception as exc:
        raise TypeError("csr_array expects (data, indices, indptr) or a CSRArray instance.") from exc
    data = ensure_array(data)
    indices = ensure_array(indices, device=data.device)
    indptr = ensure_array(indptr, device=data.device)
    if mode != "none":
        validate_csr_metadata(data, indices, indptr, shape)
    if mode == "full":
        validate_csr_values(indices, indptr, shape, data.shape[0])
    canon = bool(canonical) if canonical is not None else False
    return CSRArray(data, indices, indptr, shape, sorted_indices=sorted_indices or canon, has_canonical_format=canon)
