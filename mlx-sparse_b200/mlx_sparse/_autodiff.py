"""Autograd of the sparse products (torch.autograd).

The reference differentiates ``csr_matvec`` / ``csr_matmul`` with respect to
the stored values and the dense right-hand side (``src/sparse/csr_matvec/
csr_matvec.cpp:236-263``: VJP = ``csr_matvec_data_vjp`` for the values and
``csr_matvec_transpose`` for x; the same pair for ``csr_matmul``). Here the
value cotangent runs in ``msx_csr_*_data_vjp`` and the transposed product as a
plain SpMV / SpMM over the matrix's cached transposed structure (built once by
``msx_csr_transpose``), whose rows list every column's entries in the
reference's row-major order.
"""

from __future__ import annotations

import torch

from mlx_sparse import _native


class CsrProduct(torch.autograd.Function):
    """``A @ rhs`` (rank-1 or rank-2 rhs) differentiable in ``data`` and
    ``rhs``; ``a`` supplies the structure (indices, indptr, shape)."""

    @staticmethod
    def forward(ctx, data, rhs, a):
        ctx.a = a
        ctx.save_for_backward(data, rhs)
        if rhs.ndim == 1:
            plan = a.spmv_plan() if a.shape[0] > 0 else None
            return _native.csr_matvec(data, a.indices, a.indptr, rhs, a.shape, plan=plan)
        return _native.csr_matmul(data, a.indices, a.indptr, rhs, a.shape)

    @staticmethod
    def backward(ctx, grad):
        data, rhs = ctx.saved_tensors
        a = ctx.a
        grad = grad.contiguous()
        g_data = g_rhs = None
        if ctx.needs_input_grad[0]:
            g_data = _native.csr_data_vjp(a.indices, a.indptr, rhs, grad, a.shape)
        if ctx.needs_input_grad[1]:
            indices, indptr, perm = a.transpose_structure()
            t_data = data.index_select(0, perm)
            t_shape = (a.shape[1], a.shape[0])
            if rhs.ndim == 1:
                if "t_plan" not in a._cache and t_shape[0] > 0:
                    a._cache["t_plan"] = _native.SpmvPlan(indptr, t_shape[0], indices.numel())
                g_rhs = _native.csr_matvec(t_data, indices, indptr, grad, t_shape, plan=a._cache.get("t_plan"))
            else:
                g_rhs = _native.csr_matmul(t_data, indices, indptr, grad, t_shape)
        return g_data, g_rhs, None
