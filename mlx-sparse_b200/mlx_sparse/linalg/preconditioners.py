"""Preconditioners that the native CG path accepts: identity, diagonal,
Jacobi and Chebyshev.

Mirrors mlx-sparse's ``mlx_sparse/linalg/preconditioners.py`` for the CG path:
``DiagonalPreconditioner`` (:150-233), ``JacobiPreconditioner`` (:247-265),
``ChebyshevPreconditioner`` (:870-985), ``identity`` (:998-1012), ``diagonal``
(:1015-1063), ``jacobi`` (:1066-1150), ``chebyshev`` (:1290-1428) and
``aspreconditioner`` (:1546-1584). Setup runs on the device and synchronises
for the reference's validation checks (finite / near-zero diagonal, spectral
bounds), exactly where the reference reads values back to the host. Applying
a diagonal or Chebyshev preconditioner (``solve``) runs in the CUDA library
(``msx_diagonal_preconditioner_apply``, ``msx_csr_chebyshev_apply``).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
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
        """``inverse_diagonal * x`` for ``x`` of shape ``(n,)`` or ``(n, k)``
        (the reference's ``diagonal_preconditioner_apply``,
        ``src/preconditioners/diagonal/diagonal.cpp:60-88``)."""
        from mlx_sparse import _native

        x = ensure_array(x, device=self.inverse_diagonal.device)
        if x.ndim not in (1, 2):
            raise ValueError("diagonal_preconditioner_apply rhs must be rank-1 or rank-2.")
        if x.shape[0] != self.shape[0]:
            raise ValueError("diagonal_preconditioner_apply rhs leading dimension must match inv_diag length.")
        if x.dtype != torch.float32:
            raise ValueError("diagonal_preconditioner_apply rhs currently requires dtype float32.")
        return _native.diagonal_preconditioner_apply(self.inverse_diagonal, x)

    matvec = solve
    __call__ = solve


@dataclass(frozen=True)
class JacobiPreconditioner(DiagonalPreconditioner):
    kind: str = "jacobi"
    omega: float = 1.0
    shift: float = 0.0
    zero_policy: str = "raise"
    zero_atol: float = 0.0
    checked: bool = False
    positive_diagonal: bool | None = None


@dataclass(frozen=True)
class ChebyshevPreconditioner:
    """Fixed-degree first-kind Chebyshev polynomial preconditioner on a square
    fp32 CSR operator over the spectral interval [lambda_min, lambda_max]."""

    A: CSRArray
    degree: int = 2
    lambda_min: float = 0.0
    lambda_max: float = 0.0
    estimate: bool = True
    spectral_info: dict = None
    kind: str = "chebyshev"
    is_symmetric: bool = True
    is_positive_definite: bool = True

    def __post_init__(self) -> None:
        shape = _square_shape(self.A.shape)
        if self.A.data.dtype != torch.float32:
            raise TypeError("Chebyshev preconditioners require float32 CSR values.")
        degree = int(self.degree)
        if degree <= 0:
            raise ValueError("degree must be positive.")
        lmin = _finite_scalar("lambda_min", self.lambda_min)
        lmax = _finite_scalar("lambda_max", self.lambda_max)
        if lmin <= 0.0 or lmax <= lmin:
            raise ValueError("Chebyshev spectral interval must satisfy 0 < lambda_min < lambda_max.")
        object.__setattr__(self, "degree", degree)
        object.__setattr__(self, "lambda_min", lmin)
        object.__setattr__(self, "lambda_max", lmax)
        object.__setattr__(self, "spectral_info", dict(self.spectral_info or {}))
        if shape != self.A.shape:
            raise ValueError("Chebyshev operator shape must be square.")

    @property
    def shape(self):
        return self.A.shape

    @property
    def dtype(self):
        return torch.float32

    @property
    def nnz(self) -> int:
        return int(self.A.nnz)

    def solve(self, x):
        """``p_d(A) x`` for ``x`` of shape ``(n,)`` or ``(n, k)``
        (``csr_chebyshev_preconditioner_apply``)."""
        from mlx_sparse import _native

        x = ensure_array(x, device=self.A.device)
        if x.ndim not in (1, 2) or x.shape[0] != self.shape[0]:
            raise ValueError(f"Chebyshev apply expects a right-hand side with leading dimension {self.shape[0]}.")
        x = x.to(torch.float32)
        if not bool(torch.isfinite(x).all().item()):
            raise ValueError("right-hand side must contain only finite values.")
        return _native.csr_chebyshev_preconditioner_apply(self.A.data, self.A.indices, self.A.indptr, x, self.shape,
                                                          degree=self.degree, lambda_min=self.lambda_min,
                                                          lambda_max=self.lambda_max)

    matvec = solve
    __call__ = solve


_LANCZOS_STEPS = 20  # kDefaultEstimateSteps, src/preconditioners/chebyshev/chebyshev.cpp:41


def _jacobi_symmetric_values(a: np.ndarray) -> np.ndarray:
    """Eigenvalues of a small symmetric float32 matrix by cyclic-pivot Jacobi
    rotations (restates ``jacobi_symmetric``, ``src/linalg/common/common.h:
    259-313``: largest off-diagonal pivot, stop at 1e-6)."""
    a = np.array(a, dtype=np.float32)
    n = a.shape[0]
    iu = np.triu_indices(n, 1)
    for _ in range(max(32, 12 * n * n)):
        if n < 2:
            break
        off = np.abs(a[iu])
        k = int(np.argmax(off))
        if off[k] <= np.float32(1e-6):
            break
        p, q = int(iu[0][k]), int(iu[1][k])
        app, aqq, apq = a[p, p], a[q, q], a[p, q]
        tau = np.float32((aqq - app) / (np.float32(2.0) * apq))
        t = np.float32((np.float32(1.0) if tau >= 0 else np.float32(-1.0)) /
                       (abs(tau) + np.sqrt(np.float32(1.0) + tau * tau)))
        c = np.float32(np.float32(1.0) / np.sqrt(np.float32(1.0) + t * t))
        s = np.float32(t * c)
        cp, cq = a[:, p].copy(), a[:, q].copy()
        a[:, p], a[:, q] = c * cp - s * cq, s * cp + c * cq
        rp, rq = a[p, :].copy(), a[q, :].copy()
        a[p, :], a[q, :] = c * rp - s * rq, s * rp + c * rq
    return np.diag(a).astype(np.float32)


def _lanczos_ritz_bounds(csr: CSRArray, steps: int):
    """(ritz_min, ritz_max, used) of ``steps`` Lanczos steps with full
    reorthogonalisation from the normalised ones vector (restates
    ``host_lanczos_operator``, ``src/linalg/common/common.h:345-410``, and
    ``lanczos_ritz_bounds``, ``chebyshev.cpp:163-203``). Products run in the
    CUDA SpMV; the vector updates are fp32 with fp64 inner products."""
    n = csr.shape[0]
    steps = min(n, steps)
    if steps <= 0:
        return float("nan"), float("nan"), 0
    dev = csr.device
    basis = torch.zeros((steps, n), dtype=torch.float32, device=dev)
    basis[0] = 1.0 / float(np.sqrt(np.float32(n)))
    alphas, betas = [], []
    beta_prev = 0.0
    used = 0
    eps = float(np.finfo(np.float32).eps)
    for j in range(steps):
        q = basis[j]
        w = csr @ q
        if j > 0:
            w = w - np.float32(beta_prev) * basis[j - 1]
        alpha = float(torch.dot(q.double(), w.double()).item())
        alphas.append(np.float32(alpha))
        w = w - np.float32(alpha) * q
        for _ in range(2):
            for col in range(j + 1):
                coeff = float(torch.dot(basis[col].double(), w.double()).item())
                w = w - np.float32(coeff) * basis[col]
        beta = float(np.float32(np.sqrt(max(float(torch.dot(w.double(), w.double()).item()), 0.0))))
        betas.append(np.float32(beta))
        used = j + 1
        if j + 1 == steps or beta <= eps:
            break
        basis[j + 1] = w / np.float32(beta)
        beta_prev = beta
    tri = np.zeros((used, used), dtype=np.float32)
    for i in range(used):
        tri[i, i] = alphas[i]
        if i > 0:
            tri[i, i - 1] = tri[i - 1, i] = betas[i - 1]
    values = _jacobi_symmetric_values(tri)
    values = values[np.isfinite(values)]
    if values.size == 0:
        return float("nan"), float("nan"), used
    return float(values.min()), float(values.max()), used


def spectral_bounds(csr: CSRArray, *, estimate: bool = True, estimate_steps: int = 0):
    """``(gershgorin_min, gershgorin_max, ritz_min, ritz_max, diagonal_min,
    diagonal_max, estimate_steps)`` as the reference's
    ``csr_chebyshev_spectral_bounds`` (``chebyshev.cpp:374-425``)."""
    from mlx_sparse import _native

    if estimate_steps < 0:
        raise ValueError("csr_chebyshev_spectral_bounds estimate_steps must be non-negative.")
    gmin, gmax, dmin, dmax = _native.csr_gershgorin_bounds(csr.data, csr.indices, csr.indptr, csr.shape)
    if estimate:
        rmin, rmax, used = _lanczos_ritz_bounds(csr, estimate_steps or _LANCZOS_STEPS)
    else:
        rmin, rmax, used = float("nan"), float("nan"), 0
    return gmin, gmax, rmin, rmax, dmin, dmax, used


def chebyshev(A, *, degree: int = 2, lambda_min: float | None = None, lambda_max: float | None = None,
              estimate: bool = True) -> ChebyshevPreconditioner:
    """Chebyshev polynomial preconditioner of canonical fp32 ``A``; missing
    bounds come from the Gershgorin interval, else from Lanczos Ritz values
    (upper 1.1 x, lower max(tiny, min(0.5 x ritz_min, 0.1 x lambda_max))), as
    the reference's ``chebyshev()`` chooses them."""
    degree_value = int(degree)
    if degree_value <= 0:
        raise ValueError("degree must be positive.")
    csr = A.tocsr(canonical=True) if isinstance(A, COOArray) else A
    if not isinstance(csr, CSRArray):
        raise TypeError(f"chebyshev expects a sparse matrix, got {type(A).__name__}.")
    csr = csr.canonicalize()
    if csr.data.dtype != torch.float32:
        csr = csr.astype(torch.float32)
    if csr.shape[0] != csr.shape[1]:
        raise ValueError(f"chebyshev requires a square matrix, got {csr.shape}.")
    gmin, gmax, rmin, rmax, dmin, dmax, steps = spectral_bounds(csr, estimate=bool(estimate))

    def positive_finite(v) -> bool:
        return math.isfinite(float(v)) and float(v) > 0.0

    if lambda_max is None:
        if positive_finite(gmax):
            lmax, lmax_src = float(gmax), "gershgorin"
        elif estimate and positive_finite(rmax):
            lmax, lmax_src = 1.1 * float(rmax), "lanczos_1.1"
        else:
            raise ValueError("could not determine a positive Chebyshev upper spectral bound; pass lambda_max "
                             "explicitly.")
    else:
        lmax, lmax_src = _finite_scalar("lambda_max", lambda_max), "explicit"
    tiny = max(1.0e-12, 16.0 * 1.1920928955078125e-7)
    if lambda_min is None:
        if positive_finite(gmin):
            lmin, lmin_src = float(gmin), "gershgorin"
        elif estimate and positive_finite(rmin):
            lmin, lmin_src = max(tiny, min(0.5 * float(rmin), 0.1 * lmax)), "lanczos_0.5"
        else:
            raise ValueError("could not determine a positive Chebyshev lower spectral bound; pass lambda_min "
                             "explicitly or use estimate=True for SPD matrices whose Gershgorin lower bound is "
                             "non-positive.")
    else:
        lmin, lmin_src = _finite_scalar("lambda_min", lambda_min), "explicit"
    if not math.isfinite(lmin) or not math.isfinite(lmax) or lmin <= 0.0 or lmax <= lmin:
        raise ValueError("Chebyshev spectral interval must satisfy 0 < lambda_min < lambda_max.")
    info = {"gershgorin_min": gmin, "gershgorin_max": gmax, "ritz_min": rmin, "ritz_max": rmax,
            "diagonal_min": dmin, "diagonal_max": dmax, "estimate_steps": int(steps),
            "lambda_min_source": lmin_src, "lambda_max_source": lmax_src}
    return ChebyshevPreconditioner(A=csr, degree=degree_value, lambda_min=lmin, lambda_max=lmax,
                                   estimate=bool(estimate), spectral_info=info)


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
    if isinstance(M, (IdentityPreconditioner, DiagonalPreconditioner, ChebyshevPreconditioner)):
        if A is not None and M.shape != _square_shape(A):
            raise ValueError(f"preconditioner shape {M.shape} does not match A.shape.")
        return M
    if isinstance(M, (CSRArray, COOArray)):
        raise TypeError(
            "sparse matrices are not inverse-apply preconditioners; use "
            "preconditioners.jacobi(A) or preconditioners.diagonal(...)."
        )
    raise TypeError(
        "cg currently supports only identity, diagonal, Jacobi and Chebyshev native-backed preconditioners."
    )
