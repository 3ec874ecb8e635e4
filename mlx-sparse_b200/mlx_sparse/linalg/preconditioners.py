"""Preconditioners that the native CG path accepts: identity, diagonal, Jacobi.

Mirrors mlx-sparse's ``mlx_sparse/linalg/preconditioners.py`` for the CG path:
``DiagonalPreconditioner`` (:150-233), ``JacobiPreconditioner`` (:247-265),
``identity`` (:998-1012), ``diagonal`` (:1015-1063), ``jacobi`` (:1066-1150)
and ``aspreconditioner`` (:1546-1584). Setup runs with torch ops on the device
and synchronises for the reference's validation checks (finite / near-zero
diagonal), exactly where the reference calls ``host_bool``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from mlx_sparse._coo import COOArray
from mlx_sparse._csr import CSRArray
from mlx_sparse._validation import ensure_array


def _square_shape(A_or_shape) -> tuple[int, int]:
    if isinstance(A_or_shape, (CSRArray, COOArray)):
        shape = A_or_shape.shape
    elif isinstance(A_or_shape, int):
        shape = (A_or_shape, A_or_shape)
    else:
        shape = tuple(int(s) for s in A_or_shape)
    if len(shape) != 2 or shape[0] != shape[1]:
        raise ValueError(f"preconditioners require a square shape, got {shape}.")
    return shape


def _finite_scalar(name: str, value) -> float:
    v = float(value)
    if not math.isfinite(v):
        raise ValueError(f"{name} must be finite.")
    return v


def _float32_vector(name: str, value, *, require_finite: bool = False) -> torch.Tensor:
    v = ensure_array(value)
    if v.ndim != 1:
        raise ValueError(f"{name} must be rank-1, got shape={tuple(v.shape)}.")
    if v.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise TypeError(f"{name} must have a floating dtype, got {v.dtype}.")
    v = v.to(torch.float32).contiguous()
    if require_finite and not bool(torch.isfinite(v).all().item()):
        raise ValueError(f"{name} must contain only finite values.")
    return v


@dataclass(frozen=True)
class IdentityPreconditioner:
    shape: tuple
    dtype: object = None
    kind: str = "identity"

    def solve(self, x):
        return ensure_array(x)


@dataclass(frozen=True)
class DiagonalPreconditioner:
    """Explicit inverse-diagonal preconditioner (float32, finite)."""

    inverse_diagonal: torch.Tensor
    shape: tuple
    kind: str = "diagonal"
    is_symmetric: bool = True
    is_positive_definite: bool = False

    def __post_init__(self) -> None:
        shape = _square_shape(self.shape)
        inv = _float32_vector("inverse_diagonal", self.inverse_diagonal, require_finite=True)
        if inv.shape[0] != shape[0]:
            raise ValueError(f"inverse_diagonal has length {inv.shape[0]}, expected {shape[0]}.")
        object.__setattr__(self, "shape", shape)
        object.__setattr__(self, "inverse_diagonal", inv)

    @property
    def dtype(self):
        return self.inverse_diagonal.dtype

    @property
    def nnz(self) -> int:
        return int(self.inverse_diagonal.shape[0])

    def solve(self, x):
        x = ensure_array(x, device=self.inverse_diagonal.device)
        if x.ndim == 2:
            return self.inverse_diagonal[:, None] * x
        return self.inverse_diagonal * x

    matvec = solve


@dataclass(frozen=True)
class JacobiPreconditioner(DiagonalPreconditioner):
    kind: str = "jacobi"
    omega: float = 1.0
    shift: float = 0.0
    zero_policy: str = "raise"
    zero_atol: float = 0.0
    checked: bool = False
    positive_diagonal: bool | None = None


def identity(A_or_shape, *, dtype=None) -> IdentityPreconditioner:
    if dtype not in (None, torch.float32):
        raise TypeError("identity preconditioners currently use float32 values.")
    return IdentityPreconditioner(shape=_square_shape(A_or_shape), dtype=dtype)


def diagonal(inv_diag_or_diag, *, inverse: bool = False, shape=None, dtype=None, zero_atol: float = 0.0):
    values = _float32_vector("diagonal", inv_diag_or_diag, require_finite=True)
    if dtype not in (None, torch.float32):
        raise TypeError("diagonal preconditioners currently use float32 values.")
    pc_shape = _square_shape(shape if shape is not None else (values.shape[0], values.shape[0]))
    if inverse:
        inv = values
    else:
        if bool((values.abs() <= float(zero_atol)).any().item()):
            raise ValueError("diagonal contains zero or near-zero entries.")
        inv = 1.0 / values
    return DiagonalPreconditioner(inv, pc_shape)


def jacobi(A, *, omega: float = 1.0, shift: float = 0.0, zero_policy: str = "raise", zero_atol: float = 0.0,
           check: bool = False) -> JacobiPreconditioner:
    """``inv_diag = omega / (diag(A) + shift)`` from the canonical CSR diagonal."""
    if zero_policy not in {"raise", "unit"}:
        raise ValueError("zero_policy must be 'raise' or 'unit'.")
    omega_v = _finite_scalar("omega", omega)
    shift_v = _finite_scalar("shift", shift)
    checked = bool(check)
    if checked and omega_v <= 0.0:
        raise ValueError("omega must be positive when check=True.")
    csr = A.tocsr(canonical=True) if isinstance(A, COOArray) else A
    if not isinstance(csr, CSRArray):
        raise TypeError(f"jacobi expects a sparse matrix, got {type(A).__name__}.")
    csr = csr.canonicalize()
    if csr.shape[0] != csr.shape[1]:
        raise ValueError(f"jacobi requires a square matrix, got {csr.shape}.")
    diag = csr.diagonal().to(torch.float32)
    shifted = diag + torch.tensor(shift_v, dtype=torch.float32, device=diag.device)
    if not bool(torch.isfinite(shifted).all().item()):
        raise ValueError("shifted diagonal must contain only finite values.")
    atol = float(zero_atol)
    if atol < 0.0:
        raise ValueError("zero_atol must be non-negative.")
    near_zero = shifted.abs() <= atol
    positive = bool((shifted > atol).all().item()) if checked else None
    if bool(near_zero.any().item()):
        if zero_policy == "raise":
            raise ValueError("Jacobi shifted diagonal contains zero or near-zero entries.")
        shifted = torch.where(near_zero, torch.ones_like(shifted), shifted)
    if checked and not positive:
        raise ValueError("Jacobi shifted diagonal must be strictly positive when check=True.")
    inv = torch.tensor(omega_v, dtype=torch.float32, device=shifted.device) / shifted
    return JacobiPreconditioner(inv, csr.shape, is_positive_definite=checked, omega=omega_v, shift=shift_v,
                                zero_policy=zero_policy, zero_atol=atol, checked=checked,
                                positive_diagonal=positive)


def aspreconditioner(M, A=None):
    if M is None:
        if A is None:
            raise ValueError("A is required when M is None.")
        return identity(A)
    if isinstance(M, (IdentityPreconditioner, DiagonalPreconditioner)):
        if A is not None and M.shape != _square_shape(A):
            raise ValueError(f"preconditioner shape {M.shape} does not match A.shape.")
        return M
    if isinstance(M, (CSRArray, COOArray)):
        raise TypeError(
            "sparse matrices are not inverse-apply preconditioners; use "
            "preconditioners.jacobi(A) or preconditioners.diagonal(...)."
        )
    raise TypeError(
        "cg currently supports only identity, diagonal and Jacobi native-backed preconditioners."
    )
