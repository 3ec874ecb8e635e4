"""mlx_sparse - B200 (sm_100a) build of mlx-sparse's sparse-product path.

Drop-in for the reference's ``csr_array`` / ``coo_array`` containers and their
products (``a @ x`` SpMV, ``a @ B`` SpMM, ``a @ b_sparse`` SpGEMM) and for
``linalg.cg`` (plain and Jacobi-preconditioned), with torch CUDA tensors in
place of MLX arrays. Every product runs in the hand-written CUDA library
``_lib/libmsx_b200.so``; there is no CPU fallback.
"""

from mlx_sparse import linalg
from mlx_sparse._coo import COOArray, coo_array
from mlx_sparse._csr import CSRArray, csr_array
from mlx_sparse._native import check_device_errors, extension, library_path
from mlx_sparse._ops import (
    coo_matmat,
    coo_matmul,
    coo_matvec,
    csr_batched_matmul,
    csr_batched_matvec,
    csr_matmat,
    csr_matmul,
    csr_matmul_data_vjp,
    csr_matmul_streamed,
    csr_matmul_transpose,
    csr_matvec,
    csr_matvec_data_vjp,
    csr_matvec_transpose,
)

__version__ = "0.1.0"

__all__ = [
    "COOArray",
    "CSRArray",
    "check_device_errors",
    "coo_array",
    "coo_matmat",
    "coo_matmul",
    "coo_matvec",
    "csr_array",
    "csr_matmat",
    "csr_batched_matmul",
    "csr_batched_matvec",
    "csr_matmul",
    "csr_matmul_data_vjp",
    "csr_matmul_streamed",
    "csr_matmul_transpose",
    "csr_matvec",
    "csr_matvec_data_vjp",
    "csr_matvec_transpose",
    "extension",
    "library_path",
    "linalg",
]
