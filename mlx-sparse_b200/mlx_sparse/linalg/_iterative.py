"""``cg``: the conjugate-gradient driver over the native solve.

Mirrors mlx-sparse's ``mlx_sparse/linalg/_iterative.py`` ``cg`` (:69-325) on the
native path: the matrix is normalised to canonical float32 CSR, ``b``/``x0`` to
float32 vectors, ``maxiter`` defaults to ``10 * n``
(``linalg/utils/iterative.py:49-70``), and the solve dispatches to
``csr_cg`` (M None / identity) or ``csr_pcg_jacobi`` (diagonal / Jacobi). The
whole Krylov loop runs on the GPU; Python sees only the final status
(``finish_solver_result``, ``linalg/utils/diagnostics/callbacks.py:61-101``).
"""

from __future__ import annotations

import torch

from mlx_sparse import _native
from mlx_sparse._coo import COOArray
from mlx_sparse._csr import CSRArray
from mlx_sparse._validation import ensure_array
from mlx_sparse.linalg import preconditioners
from mlx_sparse.linalg.diagnostics import finish_solver_result


def _as_csr(A) -> CSRArray:
    if isinstance(A, COOArray):
        return A.tocsr(canonical=True)
    if isinstance(A, CSRArray):
        return A.canonicalize()
    if isinstance(A, torch.Tensor):
        raise TypeError("sparse iterative solvers expect a sparse matrix; use torch.linalg for dense arrays.")
    raise TypeError(f"sparse iterative solvers expect a sparse matrix, got {type(A).__name__}.")


def _float32_csr(csr: CSRArray) -> CSRArray:
    if csr.data.dtype == torch.float32:
        return csr
    if csr.data.dtype in (torch.float16, torch.bfloat16):
        return csr.astype(torch.float32)
    raise TypeError(f"sparse iterative solvers require float32 values, got {csr.data.dtype}.")


def _float32_array(x, device) -> torch.Tensor:
    t = ensure_array(x, device=device)
    if t.dtype in (torch.float16, torch.bfloat16, torch.float64):
        t = t.to(torch.float32)
    if t.dtype != torch.float32:
        raise TypeError(f"sparse iterative solvers require float32 vectors, got {t.dtype}.")
    return t.contiguous()


def _guess(csr: CSRArray, b: torch.Tensor, x0) -> torch.Tensor:
    if b.ndim != 1:
        raise ValueError(f"right-hand side must be rank-1, got {tuple(b.shape)}.")
    if b.shape[0] != csr.shape[0]:
        raise ValueError(f"b has length {b.shape[0]}, expected {csr.shape[0]}.")
    if x0 is None:
        return torch.zeros(csr.shape[1], dtype=torch.float32, device=b.device)
    x = _float32_array(x0, b.device)
    if x.ndim != 1 or x.shape[0] != csr.shape[1]:
        raise ValueError(f"x0 must have shape ({csr.shape[1]},), got {tuple(x.shape)}.")
    return x


def _maxiter(csr: CSRArray, maxiter) -> int:
    value = 10 * csr.shape[1] if maxiter is None else int(maxiter)
    if value < 0:
        raise ValueError("maxiter must be non-negative.")
    return value


def _solve(csr: CSRArray, rhs, guess, inv_diag, rtol, atol, maxiter):
    """Native solve. Square matrices reuse the matrix's cached solver context
    (same recurrence as ``_native.csr_cg`` / ``csr_pcg_jacobi``, setup paid
    once per matrix); otherwise the stateless entry points validate and raise
    exactly as the reference's primitives do."""
    n_rows, n_cols = csr.shape
    if n_rows > 0 and n_rows == n_cols and rhs.shape[0] == n_rows:
        ctx = csr.cg_context(inv_diag is not None)
        return ctx.solve(rhs, guess, inv_diag, rtol=float(rtol), atol=float(atol), maxiter=maxiter)
    if inv_diag is not None:
        return _native.csr_pcg_jacobi(csr.data, csr.indices, csr.indptr, rhs, guess, inv_diag, csr.shape,
                                      rtol=float(rtol), atol=float(atol), maxiter=maxiter)
    return _native.csr_cg(csr.data, csr.indices, csr.indptr, rhs, guess, csr.shape, rtol=float(rtol),
                          atol=float(atol), maxiter=maxiter)


def cg(A, b, *, x0=None, rtol: float = 1e-5, atol: float = 0.0, maxiter: int | None = None, M=None,
       callback=None, return_info: bool = False):
    """Solves the SPD system ``A x = b`` with (Jacobi-preconditioned) CG.

    Stops when ``||r|| <= max(atol, rtol * ||b||)``. Returns ``(x, info)``:
    ``info == 0`` converged, ``> 0`` iteration budget exhausted, ``< 0``
    breakdown (-1), non-positive preconditioned product (-2) or non-finite
    value (-3). ``return_info=True`` returns a ``SolverInfo`` instead.
    """
    csr = _float32_csr(_as_csr(A))
    rhs = _float32_array(b, csr.device)
    guess = _guess(csr, rhs, x0)
    maxiter_value = _maxiter(csr, maxiter)
    kind = None
    if M is not None:
        pc = preconditioners.aspreconditioner(M, csr)
        kind = pc.kind
        if isinstance(pc, preconditioners.ChebyshevPreconditioner):
            # csr_pcg_chebyshev, as the reference dispatches it (mlx_sparse/linalg/_iterative.py:266-283)
            Mc = pc.A
            if Mc.device != csr.device:
                raise ValueError("the Chebyshev preconditioner must live on the matrix's device.")
            if Mc.indices.dtype != csr.indices.dtype:
                Mc = type(Mc)(Mc.data, Mc.indices.to(csr.indices.dtype), Mc.indptr.to(csr.indices.dtype), Mc.shape,
                              Mc.sorted_indices, Mc.has_canonical_format)
            x, info, residual, iterations = _native.csr_pcg_chebyshev(
                csr.data, csr.indices, csr.indptr, rhs, guess, (Mc.data, Mc.indices, Mc.indptr), csr.shape,
                degree=pc.degree, lambda_min=pc.lambda_min, lambda_max=pc.lambda_max, rtol=float(rtol),
                atol=float(atol), maxiter=maxiter_value)
            return finish_solver_result(x, info, residual, iterations, solver="cg", return_info=bool(return_info),
                                        callback=callback, rtol=float(rtol), atol=float(atol),
                                        maxiter=maxiter_value, preconditioner=kind)
        if isinstance(pc, preconditioners.DiagonalPreconditioner):
            x, info, residual, iterations = _solve(csr, rhs, guess, pc.inverse_diagonal.to(csr.device),
                                                   rtol, atol, maxiter_value)
            return finish_solver_result(x, info, residual, iterations, solver="cg", return_info=bool(return_info),
                                        callback=callback, rtol=float(rtol), atol=float(atol),
                                        maxiter=maxiter_value, preconditioner=kind)
    x, info, residual, iterations = _solve(csr, rhs, guess, None, rtol, atol, maxiter_value)
    return finish_solver_result(x, info, residual, iterations, solver="cg", return_info=bool(return_info),
                                callback=callback, rtol=float(rtol), atol=float(atol), maxiter=maxiter_value,
                                preconditioner=kind)
