"""Native seam: ctypes bindings of the sm_100a C-ABI library ``libmsx_b200.so``.

Mirrors mlx-sparse's ``mlx_sparse/_native.py`` (csr_matvec :179-189, csr_matmul
:286-296, csr_matmat :393-408, csr_cg :883-909, csr_pcg_jacobi :1139-1167):
same function names and argument meaning, torch CUDA tensors in place of MLX
arrays. Those five cross the boundary as DLPack tensors (``msx_dl_*``: each
argument is the ``DLTensor`` of a ``torch.utils.dlpack`` capsule, kept alive
for the call), as the reference hands device arrays to its native module; the
other entry points take raw device pointers. There is no CPU fallback: if the
library or a CUDA device is missing, every op raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes
import os
import threading

import torch
from torch.utils.dlpack import to_dlpack

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "_lib", "libmsx_b200.so")

MSX_F32, MSX_F16, MSX_BF16 = 0, 1, 2
MSX_I32, MSX_I64 = 0, 1

VALUE_CODES = {torch.float32: MSX_F32, torch.float16: MSX_F16, torch.bfloat16: MSX_BF16}
INDEX_CODES = {torch.int32: MSX_I32, torch.int64: MSX_I64}

_ERRORS = {1: ValueError, 2: TypeError, 3: OverflowError, 4: RuntimeError, 5: RuntimeError}

_lib = None
_lib_lock = threading.Lock()


def library_path() -> str:
    return LIB_PATH


def extension():
    """Loads the CUDA library; raises RuntimeError when it is unavailable."""
    global _lib
    if _lib is not None:
        return _lib
    with _lib_lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"mlx_sparse CUDA library not found at {LIB_PATH}; build it with "
                "`python mlx-sparse_b200/build.py` (there is no CPU fallback)."
            )
        L = ctypes.CDLL(LIB_PATH)
        p, i64, c_int, c_float = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
        L.msx_last_error.restype = ctypes.c_char_p
        L.msx_spmv_plan_create.argtypes = [c_int, p, i64, i64, p, ctypes.POINTER(p)]
        L.msx_spmv_plan_destroy.argtypes = [p]
        L.msx_spmv_plan_info.argtypes = [p, ctypes.POINTER(i64), ctypes.POINTER(i64)]
        L.msx_csr_matvec.argtypes = [c_int, c_int, p, p, p, i64, p, p, i64, i64, p, p]
        L.msx_csr_matmul.argtypes = [c_int, c_int, p, p, p, i64, p, i64, p, i64, i64, p]
        L.msx_csr_batched_matvec.argtypes = [c_int, c_int, p, p, p, i64, p, i64, p, i64, i64, p]
        L.msx_csr_batched_matmul.argtypes = [c_int, c_int, p, p, p, i64, p, i64, i64, p, i64, i64, p]
        mm = [c_int, c_int, p, p, p, i64, c_int, p, p, p, i64, i64, i64, i64, i64, c_int]
        if hasattr(L, "msx_csr_matmat_symbolic"):
            L.msx_csr_matmat_symbolic.argtypes = mm + [p, ctypes.POINTER(i64), c_int, p]
            L.msx_csr_matmat_numeric.argtypes = mm + [p, i64, p, p, c_int, p]
        if hasattr(L, "msx_csr_cg"):
            L.msx_csr_cg.argtypes = [c_int, p, p, p, i64, p, p, p, i64, i64, c_float, c_float, ctypes.c_int32,
                                     p, p, p, p]
            L.msx_csr_pcg_jacobi.argtypes = [c_int, p, p, p, i64, p, p, p, p, i64, i64, c_float, c_float,
                                             ctypes.c_int32, p, p, p, p]
        L.msx_csr_diagonal.argtypes = [c_int, c_int, p, p, p, i64, i64, i64, p, p]
        L.msx_check_device_errors.argtypes = [p]
        L.msx_debug_set_spmv_poll_limit.argtypes = [i64]
        L.msx_coo_tocsr.argtypes = [c_int, c_int, p, p, p, i64, i64, i64, c_int, p, p, p, p, p]
        L.msx_csr_transpose.argtypes = [c_int, c_int, p, p, p, i64, i64, i64, p, p, p, p, p]
        L.msx_csr_matvec_transpose.argtypes = [c_int, c_int, p, p, p, i64, p, p, i64, i64, p]
        L.msx_csr_matmul_transpose.argtypes = [c_int, c_int, p, p, p, i64, p, i64, p, i64, i64, p]
        L.msx_csr_matvec_data_vjp.argtypes = [c_int, c_int, p, p, i64, p, p, p, i64, i64, p]
        L.msx_csr_matmul_data_vjp.argtypes = [c_int, c_int, p, p, i64, p, p, i64, p, i64, i64, p]
        L.msx_csr_pcg_chebyshev.argtypes = [c_int, p, p, p, i64, p, p, p, p, p, i64, p, i64, i64, ctypes.c_int32,
                                            c_float, c_float, c_float, c_float, ctypes.c_int32, p, p, p, p]
        L.msx_csr_chebyshev_apply.argtypes = [c_int, p, p, p, i64, i64, p, i64, p, ctypes.c_int32, c_float, c_float,
                                              p]
        L.msx_diagonal_preconditioner_apply.argtypes = [p, p, i64, i64, p, p]
        L.msx_csr_gershgorin_bounds.argtypes = [c_int, p, p, p, i64, i64, i64, p, p]
        L.msx_cg_context_create.argtypes = [c_int, p, p, p, i64, i64, i64, c_int, c_int, c_int, c_int, p, c_int, p,
                                            p, p, p, p, p, ctypes.POINTER(p)]
        L.msx_cg_context_ipc_handles.argtypes = [p, p, i64]
        L.msx_cg_context_connect.argtypes = [p, p, i64]
        L.msx_cg_context_solve.argtypes = [p, p, p, p, p, c_float, c_float, ctypes.c_int32, p, p, p, p]
        L.msx_cg_context_destroy.argtypes = [p]
        dl = [p, p, p, p, p]
        L.msx_dl_csr_matvec.argtypes = dl + [i64, i64, p, p]
        L.msx_dl_csr_matmul.argtypes = dl + [i64, i64, p]
        L.msx_dl_csr_matmat_symbolic.argtypes = [p] * 6 + [i64] * 4 + [p, ctypes.POINTER(i64), c_int, p]
        L.msx_dl_csr_matmat_numeric.argtypes = [p] * 6 + [i64] * 4 + [p, p, p, c_int, p]
        L.msx_dl_csr_cg.argtypes = [p] * 6 + [i64, i64, c_float, c_float, ctypes.c_int32, p, p, p, p]
        L.msx_dl_csr_pcg_jacobi.argtypes = [p] * 7 + [i64, i64, c_float, c_float, ctypes.c_int32, p, p, p, p]
        if hasattr(L, "msx_dist_pcg"):
            L.msx_dist_unique_id.argtypes = [p, i64]
            L.msx_dist_comm_create.argtypes = [p, c_int, c_int, ctypes.POINTER(p)]
            L.msx_dist_comm_destroy.argtypes = [p]
            L.msx_dist_pcg.argtypes = [p, c_int, p, p, p, i64, i64, i64, p, p, p, p, c_float, c_float,
                                       ctypes.c_int32, c_int, p, p, p, p, p, p, p, p]
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != 0:
        msg = extension().msx_last_error().decode()
        raise _ERRORS.get(status, RuntimeError)(msg)


def require_cuda(*tensors) -> torch.device:
    dev = None
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(
                "mlx_sparse (B200 build) runs on CUDA tensors only; got a tensor on "
                f"{t.device}. Move inputs to a CUDA device (there is no CPU fallback)."
            )
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"all inputs must be on one device, got {dev} and {t.device}.")
    return dev


def stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _p(t) -> int:
    return t.data_ptr() if t is not None else 0


_capsule_ptr = ctypes.pythonapi.PyCapsule_GetPointer
_capsule_ptr.restype = ctypes.c_void_p
_capsule_ptr.argtypes = [ctypes.py_object, ctypes.c_char_p]
_capsule_name = ctypes.pythonapi.PyCapsule_GetName
_capsule_name.restype = ctypes.c_char_p
_capsule_name.argtypes = [ctypes.py_object]
# DLManagedTensorVersioned puts {version, manager_ctx, deleter, flags} (32
# bytes) before its DLTensor; the legacy DLManagedTensor starts with it.
_VERSIONED_OFFSET = 32


class _DL:
    """DLTensor pointers of torch tensors for one native call; the capsules
    (and so the tensors' DLPack views) stay alive as long as this object."""

    __slots__ = ("caps",)

    def __init__(self):
        self.caps = []

    def __call__(self, t):
        if t is None:
            return None
        cap = to_dlpack(t.detach())
        self.caps.append(cap)
        name = _capsule_name(cap)
        ptr = _capsule_ptr(cap, name)
        return ptr + (_VERSIONED_OFFSET if name == b"dltensor_versioned" else 0)


class SpmvPlan:
    """Owns an ``msx_spmv_plan`` (row-length bins of one matrix)."""

    __slots__ = ("handle", "n_blocks", "n_long", "device", "__weakref__")

    def __init__(self, indptr: torch.Tensor, n_rows: int, nnz: int):
        L = extension()
        self.device = indptr.device
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(L.msx_spmv_plan_create(INDEX_CODES[indptr.dtype], _p(indptr), n_rows, nnz,
                                         stream_ptr(self.device), ctypes.byref(h)))
        self.handle = h
        nt, ns = ctypes.c_int64(), ctypes.c_int64()
        check(L.msx_spmv_plan_info(h, ctypes.byref(nt), ctypes.byref(ns)))
        self.n_blocks, self.n_long = nt.value, ns.value

    def __del__(self):
        try:
            if self.handle:
                # outstanding kernels may still read the plan
                torch.cuda.synchronize(self.device)
                extension().msx_spmv_plan_destroy(self.handle)
                self.handle = None
        except Exception:
            pass


def csr_matvec(data, indices, indptr, x, shape, *, plan: SpmvPlan | None = None, out=None):
    L = extension()
    dev = require_cuda(data, indices, indptr, x)
    data, indices, indptr, x = (t.contiguous() for t in (data, indices, indptr, x))
    y = out if out is not None else torch.empty(shape[0], dtype=data.dtype, device=dev)
    dl = _DL()
    with torch.cuda.device(dev):
        check(L.msx_dl_csr_matvec(dl(data), dl(indices), dl(indptr), dl(x), dl(y), shape[0], shape[1],
                                  plan.handle if plan is not None else None, stream_ptr(dev)))
    return y


def csr_matmul(data, indices, indptr, rhs, shape, *, out=None):
    L = extension()
    dev = require_cuda(data, indices, indptr, rhs)
    data, indices, indptr, rhs = (t.contiguous() for t in (data, indices, indptr, rhs))
    k = rhs.shape[1]
    y = out if out is not None else torch.empty((shape[0], k), dtype=data.dtype, device=dev)
    dl = _DL()
    with torch.cuda.device(dev):
        check(L.msx_dl_csr_matmul(dl(data), dl(indices), dl(indptr), dl(rhs), dl(y), shape[0], shape[1],
                                  stream_ptr(dev)))
    return y


def csr_batched_matvec(data, indices, indptr, rhs, shape):
    """``Y[b] = A @ X[b]`` for ``rhs`` of shape ``(batch, n_cols)``."""
    L = extension()
    dev = require_cuda(data, indices, indptr, rhs)
    data, indices, indptr, rhs = (t.contiguous() for t in (data, indices, indptr, rhs))
    batch = rhs.shape[0]
    y = torch.empty((batch, shape[0]), dtype=data.dtype, device=dev)
    with torch.cuda.device(dev):
        check(L.msx_csr_batched_matvec(VALUE_CODES[data.dtype], INDEX_CODES[indices.dtype], _p(data), _p(indices),
                                       _p(indptr), data.numel(), _p(rhs), batch, _p(y), shape[0], shape[1],
                                       stream_ptr(dev)))
    return y


def csr_batched_matmul(data, indices, indptr, rhs, shape):
    """``Y[b] = A @ B[b]`` for ``rhs`` of shape ``(batch, n_cols, k)``."""
    L = extension()
    dev = require_cuda(data, indices, indptr, rhs)
    data, indices, indptr, rhs = (t.contiguous() for t in (data, indices, indptr, rhs))
    batch, k = rhs.shape[0], rhs.shape[2]
    y = torch.empty((batch, shape[0], k), dtype=data.dtype, device=dev)
    with torch.cuda.device(dev):
        check(L.msx_csr_batched_matmul(VALUE_CODES[data.dtype], INDEX_CODES[indices.dtype], _p(data), _p(indices),
                                       _p(indptr), data.numel(), _p(rhs), batch, k, _p(y), shape[0], shape[1],
                                       stream_ptr(dev)))
    return y


def csr_matmat(lhs, rhs, *, prune_zeros: bool = True):
    """Returns (data, indices, indptr) of the canonical product lhs @ rhs."""
    L = extension()
    dev = require_cuda(lhs.data, lhs.indices, lhs.indptr, rhs.data, rhs.indices, rhs.indptr)
    ld, li, lp = (t.contiguous() for t in (lhs.data, lhs.indices, lhs.indptr))
    rd, ri, rp = (t.contiguous() for t in (rhs.data, rhs.indices, rhs.indptr))
    out_it = li.dtype if li.dtype == ri.dtype else torch.int64
    m = lhs.shape[0]
    out_indptr = torch.empty(m + 1, dtype=out_it, device=dev)
    nnz = ctypes.c_int64()
    dl = _DL()
    args = [dl(ld), dl(li), dl(lp), dl(rd), dl(ri), dl(rp), lhs.shape[0], lhs.shape[1], rhs.shape[0], rhs.shape[1]]
    with torch.cuda.device(dev):
        s = stream_ptr(dev)
        check(L.msx_dl_csr_matmat_symbolic(*args, dl(out_indptr), ctypes.byref(nnz), int(prune_zeros), s))
        out_data = torch.empty(nnz.value, dtype=ld.dtype, device=dev)
        out_indices = torch.empty(nnz.value, dtype=out_it, device=dev)
        check(L.msx_dl_csr_matmat_numeric(*args, dl(out_indptr), dl(out_data), dl(out_indices), int(prune_zeros), s))
    return out_data, out_indices, out_indptr


def csr_diagonal(data, indices, indptr, shape):
    L = extension()
    dev = require_cuda(data, indices, indptr)
    data, indices, indptr = (t.contiguous() for t in (data, indices, indptr))
    out = torch.empty(min(shape), dtype=data.dtype, device=dev)
    with torch.cuda.device(dev):
        check(L.msx_csr_diagonal(VALUE_CODES[data.dtype], INDEX_CODES[indices.dtype], _p(data), _p(indices),
                                 _p(indptr), data.numel(), shape[0], shape[1], _p(out), stream_ptr(dev)))
    return out


class CgContext:
    """A persistent CG solver (``msx_cg_context``): row bins, work buffers and
    the CUDA graph of the iterations are built once, then every ``solve``
    only runs the iterations. The matrix arrays are borrowed and must outlive
    the context."""

    COMM_NONE, COMM_NCCL, COMM_P2P = 0, 1, 2
    IPC_BYTES = 256  # MSX_CG_IPC_BYTES

    def __init__(self, data, indices, indptr, n_owned, n_halo, preconditioned, *, comm=0, rank=0, world=1,
                 nccl_comm=None, peers=None, send_counts=None, recv_counts=None, send_idx=None,
                 dst_offset=None):
        import numpy as np

        L = extension()
        self.device = data.device
        self._keep = (data, indices, indptr, send_idx)
        self._peers = np.ascontiguousarray(peers if peers is not None else [], dtype=np.int32)
        self._sc = np.ascontiguousarray(send_counts if send_counts is not None else [], dtype=np.int64)
        self._rc = np.ascontiguousarray(recv_counts if recv_counts is not None else [], dtype=np.int64)
        self._off = np.ascontiguousarray(dst_offset if dst_offset is not None else [], dtype=np.int64)
        self.n = int(n_owned)
        self.world = world
        h = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            check(L.msx_cg_context_create(
                INDEX_CODES[indices.dtype], _p(data), _p(indices), _p(indptr), data.numel(), n_owned, n_halo,
                int(bool(preconditioned)), comm, rank, world, nccl_comm, int(self._peers.shape[0]),
                self._peers.ctypes.data, self._sc.ctypes.data, self._rc.ctypes.data,
                _p(send_idx) if send_idx is not None else None,
                self._off.ctypes.data if self._off.size else None, stream_ptr(self.device), ctypes.byref(h)))
        self.handle = h

    def ipc_handles(self) -> bytes:
        buf = ctypes.create_string_buffer(self.IPC_BYTES)
        check(extension().msx_cg_context_ipc_handles(self.handle, buf, self.IPC_BYTES))
        return bytes(buf.raw)

    def connect(self, all_handles: list) -> None:
        blob = b"".join(all_handles)
        buf = ctypes.create_string_buffer(blob, len(blob))
        with torch.cuda.device(self.device):
            check(extension().msx_cg_context_connect(self.handle, buf, len(blob)))

    def solve(self, b, x0, inv_diag, *, rtol, atol, maxiter):
        dev = self.device
        b = b.to(dev, torch.float32).contiguous()
        x0 = x0.to(dev, torch.float32).contiguous()
        inv = None if inv_diag is None else inv_diag.to(dev, torch.float32).contiguous()
        x = torch.empty(self.n, dtype=torch.float32, device=dev)
        info, res, its = ctypes.c_int32(), ctypes.c_float(), ctypes.c_int32()
        with torch.cuda.device(dev):
            check(extension().msx_cg_context_solve(self.handle, _p(b), _p(x0), _p(inv), _p(x), float(rtol),
                                                   float(atol), int(maxiter), ctypes.addressof(info),
                                                   ctypes.addressof(res), ctypes.addressof(its), stream_ptr(dev)))
        return x, info.value, res.value, its.value

    def __del__(self):
        try:
            if self.handle:
                extension().msx_cg_context_destroy(self.handle)
                self.handle = None
        except Exception:
            pass


def _solver_outputs(dev, n):
    x = torch.empty(n, dtype=torch.float32, device=dev)
    return x, ctypes.c_int32(), ctypes.c_float(), ctypes.c_int32()


def csr_cg(data, indices, indptr, b, x0, shape, *, rtol, atol, maxiter):
    L = extension()
    dev = require_cuda(data, indices, indptr, b, x0)
    data, indices, indptr, b, x0 = (t.contiguous() for t in (data, indices, indptr, b, x0))
    x, info, res, its = _solver_outputs(dev, shape[0])
    dl = _DL()
    with torch.cuda.device(dev):
        check(L.msx_dl_csr_cg(dl(data), dl(indices), dl(indptr), dl(b), dl(x0), dl(x), shape[0], shape[1],
                              float(rtol), float(atol), int(maxiter), ctypes.addressof(info), ctypes.addressof(res),
                              ctypes.addressof(its), stream_ptr(dev)))
    return x, info.value, res.value, its.value


def csr_pcg_jacobi(data, indices, indptr, b, x0, inv_diag, shape, *, rtol, atol, maxiter):
    L = extension()
    dev = require_cuda(data, indices, indptr, b, x0, inv_diag)
    data, indices, indptr, b, x0, inv_diag = (t.contiguous() for t in (data, indices, indptr, b, x0, inv_diag))
    x, info, res, its = _solver_outputs(dev, shape[0])
    dl = _DL()
    with torch.cuda.device(dev):
        check(L.msx_dl_csr_pcg_jacobi(dl(data), dl(indices), dl(indptr), dl(b), dl(x0), dl(inv_diag), dl(x),
                                      shape[0], shape[1], float(rtol), float(atol), int(maxiter),
                                      ctypes.addressof(info), ctypes.addressof(res), ctypes.addressof(its),
                                      stream_ptr(dev)))
    return x, info.value, res.value, its.value


def check_device_errors(device=None) -> None:
    """Synchronises the current stream of ``device`` and raises RuntimeError if
    a bounded device-side wait gave up since the last check (the flag is
    cleared by the check)."""
    import torch

    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        check(extension().msx_check_device_errors(stream_ptr(dev)))


def coo_tocsr(data, row, col, shape, *, sort_columns: bool = True, with_perm: bool = False):
    """COO -> CSR on the device. ``sort_columns``: rows ordered by (column,
    source position) as the reference's ``coo_tocsr``; else rows keep the
    source order. Returns ``(data, indices, indptr)`` or, with ``with_perm``,
    also the int64 source position of every output entry."""
    L = extension()
    dev = require_cuda(data, row, col)
    data, row, col = (t.contiguous() for t in (data, row, col))
    if row.dtype != col.dtype:
        raise TypeError(f"coo_tocsr row and col must share an index dtype, got {row.dtype} and {col.dtype}.")
    nnz = row.numel()
    out_d = torch.empty(nnz, dtype=data.dtype, device=dev)
    out_i = torch.empty(nnz, dtype=col.dtype, device=dev)
    out_p = torch.empty(shape[0] + 1, dtype=row.dtype, device=dev)
    perm = torch.empty(nnz, dtype=torch.int64, device=dev) if with_perm else None
    with torch.cuda.device(dev):
        check(L.msx_coo_tocsr(VALUE_CODES[data.dtype], INDEX_CODES[row.dtype], _p(data), _p(row), _p(col), nnz,
                              shape[0], shape[1], int(bool(sort_columns)), _p(out_d), _p(out_i), _p(out_p),
                              _p(perm), stream_ptr(dev)))
    return (out_d, out_i, out_p, perm) if with_perm else (out_d, out_i, out_p)


def csr_transpose_structure(indices, indptr, shape):
    """Structure of A^T: ``(indices, indptr, perm)`` with ``perm[q]`` the
    position in A of A^T's entry q (so A^T's values are ``data[perm]``)."""
    L = extension()
    dev = require_cuda(indices, indptr)
    indices, indptr = indices.contiguous(), indptr.contiguous()
    nnz = indices.numel()
    out_i = torch.empty(nnz, dtype=indices.dtype, device=dev)
    out_p = torch.empty(shape[1] + 1, dtype=indptr.dtype, device=dev)
    perm = torch.empty(nnz, dtype=torch.int64, device=dev)
    with torch.cuda.device(dev):
        check(L.msx_csr_transpose(MSX_F32, INDEX_CODES[indices.dtype], None, _p(indices), _p(indptr), nnz, shape[0],
                                  shape[1], None, _p(out_i), _p(out_p), _p(perm), stream_ptr(dev)))
    return out_i, out_p, perm


def csr_matvec_transpose(data, indices, indptr, x, shape):
    """``A^T @ x`` (stateless: the transposed structure is rebuilt per call)."""
    L = extension()
    dev = require_cuda(data, indices, indptr, x)
    data, indices, indptr, x = (t.contiguous() for t in (data, indices, indptr, x))
    out = torch.empty(shape[1], dtype=data.dtype, device=dev)
    with torch.cuda.device(dev):
        check(L.msx_csr_matvec_transpose(VALUE_CODES[data.dtype], INDEX_CODES[indices.dtype], _p(data), _p(indices),
                                         _p(indptr), data.numel(), _p(x), _p(out), shape[0], shape[1],
                                         stream_ptr(dev)))
    return out


def csr_matmul_transpose(data, indices, indptr, rhs, shape):
    """``A^T @ B`` for a row-major ``B`` of shape ``(n_rows, k)``."""
    L = extension()
    dev = require_cuda(data, indices, indptr, rhs)
    data, indices, indptr, rhs = (t.contiguous() for t in (data, indices, indptr, rhs))
    k = rhs.shape[1]
    out = torch.empty((shape[1], k), dtype=data.dtype, device=dev)
    with torch.cuda.device(dev):
        check(L.msx_csr_matmul_transpose(VALUE_CODES[data.dtype], INDEX_CODES[indices.dtype], _p(data), _p(indices),
                                         _p(indptr), data.numel(), _p(rhs), k, _p(out), shape[0], shape[1],
                                         stream_ptr(dev)))
    return out


def csr_data_vjp(indices, indptr, rhs, cotangent, shape):
    """Cotangent of the stored values of ``A @ rhs``: ``out[p] =
    cot[row(p)] * x[col(p)]`` (rank-1 rhs) or the row dot products
    ``cot[row(p), :] . B[col(p), :]`` (rank-2)."""
    L = extension()
    dev = require_cuda(indices, indptr, rhs, cotangent)
    indices, indptr, rhs, cotangent = (t.contiguous() for t in (indices, indptr, rhs, cotangent))
    out = torch.empty(indices.numel(), dtype=rhs.dtype, device=dev)
    with torch.cuda.device(dev):
        if rhs.ndim == 1:
            check(L.msx_csr_matvec_data_vjp(VALUE_CODES[rhs.dtype], INDEX_CODES[indices.dtype], _p(indices),
                                            _p(indptr), indices.numel(), _p(rhs), _p(cotangent), _p(out), shape[0],
                                            shape[1], stream_ptr(dev)))
        else:
            check(L.msx_csr_matmul_data_vjp(VALUE_CODES[rhs.dtype], INDEX_CODES[indices.dtype], _p(indices),
                                            _p(indptr), indices.numel(), _p(rhs), _p(cotangent), rhs.shape[1],
                                            _p(out), shape[0], shape[1], stream_ptr(dev)))
    return out


def csr_pcg_chebyshev(data, indices, indptr, b, x0, m, shape, *, degree, lambda_min, lambda_max, rtol, atol,
                      maxiter):
    """Chebyshev-preconditioned CG; ``m`` = (data, indices, indptr) of the
    preconditioner matrix. Returns ``(x, info, residual, iterations)``."""
    L = extension()
    md, mi, mp = m
    dev = require_cuda(data, indices, indptr, b, x0, md, mi, mp)
    data, indices, indptr, b, x0, md, mi, mp = (t.contiguous() for t in (data, indices, indptr, b, x0, md, mi, mp))
    x, info, res, its = _solver_outputs(dev, shape[0])
    with torch.cuda.device(dev):
        check(L.msx_csr_pcg_chebyshev(INDEX_CODES[indices.dtype], _p(data), _p(indices), _p(indptr), data.numel(),
                                      _p(b), _p(x0), _p(md), _p(mi), _p(mp), md.numel(), _p(x), shape[0], shape[1],
                                      int(degree), float(lambda_min), float(lambda_max), float(rtol), float(atol),
                                      int(maxiter), ctypes.addressof(info), ctypes.addressof(res),
                                      ctypes.addressof(its), stream_ptr(dev)))
    return x, info.value, res.value, its.value


def csr_chebyshev_preconditioner_apply(data, indices, indptr, rhs, shape, *, degree, lambda_min, lambda_max):
    """``p_d(M) rhs`` for rank-1 or rank-2 (row-major) ``rhs``."""
    L = extension()
    dev = require_cuda(data, indices, indptr, rhs)
    data, indices, indptr, rhs = (t.contiguous() for t in (data, indices, indptr, rhs))
    k = 1 if rhs.ndim == 1 else int(rhs.shape[1])
    out = torch.empty_like(rhs, dtype=torch.float32)
    with torch.cuda.device(dev):
        check(L.msx_csr_chebyshev_apply(INDEX_CODES[indices.dtype], _p(data), _p(indices), _p(indptr), data.numel(),
                                        shape[0], _p(rhs), k, _p(out), int(degree), float(lambda_min),
                                        float(lambda_max), stream_ptr(dev)))
    return out


def diagonal_preconditioner_apply(inv_diag, rhs):
    """``inv_diag[:, None] * rhs`` (rank-1 or rank-2 ``rhs``), fp32."""
    L = extension()
    dev = require_cuda(inv_diag, rhs)
    inv_diag, rhs = inv_diag.contiguous(), rhs.contiguous()
    k = 1 if rhs.ndim == 1 else int(rhs.shape[1])
    out = torch.empty_like(rhs)
    with torch.cuda.device(dev):
        check(L.msx_diagonal_preconditioner_apply(_p(inv_diag), _p(rhs), inv_diag.numel(), k, _p(out),
                                                  stream_ptr(dev)))
    return out


def csr_gershgorin_bounds(data, indices, indptr, shape):
    """(lower, upper, diag_min, diag_max) of a square fp32 CSR matrix."""
    L = extension()
    dev = require_cuda(data, indices, indptr)
    data, indices, indptr = (t.contiguous() for t in (data, indices, indptr))
    out = (ctypes.c_float * 4)()
    with torch.cuda.device(dev):
        check(L.msx_csr_gershgorin_bounds(INDEX_CODES[indices.dtype], _p(data), _p(indices), _p(indptr),
                                          data.numel(), shape[0], shape[1], out, stream_ptr(dev)))
    return tuple(float(v) for v in out)
