"""Sparse linear algebra on the product path: ``cg`` and its preconditioners."""

from mlx_sparse.linalg import preconditioners
from mlx_sparse.linalg._iterative import cg
from mlx_sparse.linalg.diagnostics import SolverInfo

__all__ = ["cg", "preconditioners", "SolverInfo"]
