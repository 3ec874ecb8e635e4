"""Solver status codes and ``SolverInfo``.

Mirrors mlx-sparse's ``linalg/utils/diagnostics/info.py`` (``SolverInfo``),
``status.py`` (``status_reason`` :50-83) and ``callbacks.py``
(``finish_solver_result`` :61-101). The native call has already synchronised
and returned host scalars, so nothing here touches the device.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True, slots=True)
class SolverInfo:
    solver: str
    status: int
    residual_norm: float
    iterations: int
    convergence_reason: str
    breakdown_reason: str | None
    message: str
    preconditioned_residual_norm: float | None = None
    rtol: float | None = None
    atol: float | None = None
    maxiter: int | None = None
    restart: int | None = None
    preconditioner: str | None = None

    @property
    def converged(self) -> bool:
        return self.status == 0

    @property
    def info(self) -> int:
        return self.status

    def __int__(self) -> int:
        return self.status


def status_reason(status: int) -> tuple[str, str | None, str]:
    if status == 0:
        return "converged", None, "converged to the requested true-residual tolerance"
    if status > 0:
        return ("iteration_limit", None,
                "iteration budget exhausted before reaching the requested tolerance")
    if status == -1:
        return ("numerical_breakdown", "breakdown",
                "solver encountered a near-zero denominator or Krylov breakdown")
    if status == -2:
        return ("invalid_preconditioner_or_operator", "non_positive_preconditioned_inner_product",
                "solver encountered a non-positive preconditioned inner product")
    if status == -3:
        return ("non_finite", "non_finite",
                "solver encountered a non-finite scalar, vector, or preconditioner output")
    return ("numerical_breakdown", f"status_{status}",
            "solver reported an implementation-specific negative breakdown status")


def make_solver_info(*, solver, status, residual_norm, iterations, rtol=None, atol=None, maxiter=None,
                     preconditioner=None) -> SolverInfo:
    reason, breakdown, message = status_reason(int(status))
    return SolverInfo(solver=solver, status=int(status), residual_norm=float(residual_norm),
                      iterations=int(iterations), convergence_reason=reason, breakdown_reason=breakdown,
                      message=message, rtol=rtol, atol=atol, maxiter=maxiter, preconditioner=preconditioner)


def finish_solver_result(x, status, residual_norm, iterations, *, solver, return_info, callback=None, rtol=None,
                         atol=None, maxiter=None, preconditioner=None):
    if return_info or callback is not None:
        diag = make_solver_info(solver=solver, status=status, residual_norm=residual_norm, iterations=iterations,
                                rtol=rtol, atol=atol, maxiter=maxiter, preconditioner=preconditioner)
        if callback is not None:
            callback(x, diag)
        return x, (diag if return_info else diag.status)
    return x, int(status)
