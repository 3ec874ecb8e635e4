"""C-ABI library checks that need no GPU: it loads, exports every symbol that
include/msx_sparse.h declares, reports errors through status codes, and the
Python layer validates metadata with the reference's messages."""

import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared_symbols():
    text = open(os.path.join(ROOT, "include", "msx_sparse.h")).read()
    return sorted(set(re.findall(r"MSX_API\s+[\w\s\*]*?\b(msx_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from mlx_sparse import _native

    lib = _native.extension()
    names = _declared_symbols()
    assert "msx_csr_matvec" in names and "msx_csr_pcg_jacobi" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, f"declared but not exported: {missing}"


def test_library_reports_invalid_arguments_without_gpu():
    from mlx_sparse import _native

    lib = _native.extension()
    assert lib.msx_compiled_sm() == 100
    # negative shape -> MSX_ERR_INVALID with the reference's message
    rc = lib.msx_csr_matvec(0, 0, None, None, None, 0, None, None, -1, 3, None, None)
    assert rc == 1
    assert b"non-negative" in lib.msx_last_error()
    # bad dtype code -> MSX_ERR_TYPE
    rc = lib.msx_csr_matvec(7, 0, None, None, None, 0, None, None, 0, 0, None, None)
    assert rc == 2
    assert b"dtype must be one of" in lib.msx_last_error()
    with pytest.raises(ValueError):
        _native.check(1)


def test_no_cpu_fallback():
    from mlx_sparse import _native

    t = torch.zeros(3)
    with pytest.raises(RuntimeError, match="CUDA"):
        _native.require_cuda(t)


def test_validation_messages_match_reference():
    from mlx_sparse import _validation as v

    d = torch.zeros(4)
    i = torch.zeros(4, dtype=torch.int32)
    p = torch.zeros(4, dtype=torch.int32)
    v.validate_csr_metadata(d, i, p, (3, 4))
    with pytest.raises(TypeError, match="dtype must be one"):
        v.validate_csr_metadata(d.to(torch.float64), i, p, (3, 4))
    with pytest.raises(TypeError, match="same dtype"):
        v.validate_csr_metadata(d, i, p.to(torch.int64), (3, 4))
    with pytest.raises(ValueError, match="n_rows"):
        v.validate_csr_metadata(d, i, p, (4, 4))
    with pytest.raises(ValueError, match="n_cols"):
        v.validate_csr_matvec_inputs(d, i, p, torch.zeros(5), (3, 4))
    with pytest.raises(TypeError, match="same dtype"):
        v.validate_csr_matvec_inputs(d, i, p, torch.zeros(4, dtype=torch.float16), (3, 4))
    with pytest.raises(ValueError, match="rank-2"):
        v.validate_csr_matmul_inputs(d, i, p, torch.zeros(4), (3, 4))


def test_solver_status_reasons():
    from mlx_sparse.linalg.diagnostics import finish_solver_result, status_reason

    assert status_reason(0)[0] == "converged"
    assert status_reason(5)[0] == "iteration_limit"
    assert status_reason(-2)[1] == "non_positive_preconditioned_inner_product"
    x, info = finish_solver_result(None, -3, 1.0, 2, solver="cg", return_info=True)
    assert info.status == -3 and not info.converged and int(info) == -3


def test_batched_and_context_entry_points_validate_without_gpu():
    """Argument checks of the batched products and the CG context run before
    any CUDA call, so they answer with status codes on a GPU-less host."""
    from mlx_sparse import _native

    lib = _native.extension()
    # negative batch -> invalid
    rc = lib.msx_csr_batched_matvec(0, 0, None, None, None, 0, None, -1, None, 4, 4, None)
    assert rc == 1 and b"non-negative" in lib.msx_last_error()
    rc = lib.msx_csr_batched_matmul(0, 0, None, None, None, 0, None, 2, -3, None, 4, 4, None)
    assert rc == 1 and b"non-negative" in lib.msx_last_error()
    # bad value dtype code -> type error
    rc = lib.msx_csr_batched_matmul(9, 0, None, None, None, 0, None, 1, 1, None, 0, 0, None)
    assert rc == 2
    # the context needs an output handle and at most 8 ranks
    out = ctypes.c_void_p()
    rc = lib.msx_cg_context_create(0, None, None, None, 0, 4, 0, 1, 0, 0, 1, None, 0, None, None, None, None, None,
                                   None, None)
    assert rc == 1
    rc = lib.msx_cg_context_create(0, None, None, None, 0, 4, 0, 1, 2, 0, 9, None, 0, None, None, None, None, None,
                                   None, ctypes.byref(out))
    assert rc == 1 and not out.value
    # peer-memory mode needs the landing offsets when there are peers
    peers = (ctypes.c_int * 1)(1)
    counts = (ctypes.c_int64 * 1)(4)
    rc = lib.msx_cg_context_create(0, None, None, None, 0, 4, 4, 1, 2, 0, 2, None, 1, peers, counts, counts, None,
                                   None, None, ctypes.byref(out))
    assert rc == 1 and b"landing offsets" in lib.msx_last_error()
    assert lib.msx_cg_context_ipc_handles(None, None, 0) == 1


class _DLDevice(ctypes.Structure):
    _fields_ = [("device_type", ctypes.c_int32), ("device_id", ctypes.c_int32)]


class _DLDataType(ctypes.Structure):
    _fields_ = [("code", ctypes.c_uint8), ("bits", ctypes.c_uint8), ("lanes", ctypes.c_uint16)]


class _DLTensor(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("device", _DLDevice), ("ndim", ctypes.c_int32),
                ("dtype", _DLDataType), ("shape", ctypes.POINTER(ctypes.c_int64)),
                ("strides", ctypes.POINTER(ctypes.c_int64)), ("byte_offset", ctypes.c_uint64)]


def test_dlpack_structs_match_the_capsules_torch_produces():
    """The header's DLTensor is the public DLPack layout: reading a torch
    capsule through it gives back the tensor's pointer, shape and dtype."""
    from mlx_sparse import _native

    assert ctypes.sizeof(_DLTensor) == 48
    t = torch.arange(12, dtype=torch.float32).reshape(3, 4)
    dl = _native._DL()
    v = _DLTensor.from_address(dl(t))
    assert v.data + v.byte_offset == t.data_ptr()
    assert (v.ndim, v.shape[0], v.shape[1]) == (2, 3, 4)
    assert (v.dtype.code, v.dtype.bits, v.dtype.lanes) == (2, 32, 1)
    assert v.device.device_type == 1  # kDLCPU
    b = _DLTensor.from_address(dl(torch.zeros(2, dtype=torch.bfloat16)))
    assert (b.dtype.code, b.dtype.bits) == (4, 16)


def test_dlpack_entry_points_reject_host_tensors_without_gpu():
    """The DLPack entry points check the device before anything else, so a CPU
    tensor is refused with the no-fallback message (no GPU needed)."""
    from mlx_sparse import _native

    lib = _native.extension()
    dl = _native._DL()
    d, i, p = torch.ones(2), torch.tensor([0, 1], dtype=torch.int32), torch.tensor([0, 1, 2], dtype=torch.int32)
    x, y = torch.ones(2), torch.empty(2)
    rc = lib.msx_dl_csr_matvec(dl(d), dl(i), dl(p), dl(x), dl(y), 2, 2, None, None)
    assert rc == 1
    assert b"CUDA device tensor" in lib.msx_last_error() and b"no CPU fallback" in lib.msx_last_error()
    rc = lib.msx_dl_csr_matvec(None, dl(i), dl(p), dl(x), dl(y), 2, 2, None, None)
    assert rc == 1 and b"must not be null" in lib.msx_last_error()
