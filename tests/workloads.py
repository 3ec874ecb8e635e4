"""Seeded synthetic inputs for the BASELINE configurations (numpy ``default_rng``).

Shared by the tests and ``bench.py`` so the oracle and the CUDA path see the
same bytes. All matrices are canonical CSR (sorted, duplicate-free rows).

- ``lap2d(m)``: 2D 5-point Laplacian on an m x m grid (node ``i*m+j``; diagonal
  4, off-diagonals -1), the SpMV config at m = 1024.
- ``poisson3d(m)``: 3D 7-point Poisson on an m^3 grid (node ``(i*m+j)*m+k``;
  diagonal 6, off-diagonals -1), the CG config at m = 256.
- ``random_k_per_row(n_rows, n_cols, k, seed)``: exactly k distinct uniform
  columns per row, values N(0,1): the SpMM (k=16, n=2^20) and SpGEMM
  (k=8, n=2^18) configs.
- ``power_law(n, seed)``: row lengths from a discrete Lomax (Pareto II) law with
  shape alpha = 2.1, min 1, capped at 65,536, scale tuned for a mean near 20;
  distinct uniform columns; values U(-1, 1): the power-law SpMV config.
"""

from __future__ import annotations

import numpy as np


def _stencil_csr(n: int, offsets_and_masks, diag_value: float, off_value: float, index_dtype):
    cols, vals, valid = [], [], []
    node = np.arange(n, dtype=np.int64)
    for off, mask in offsets_and_masks:
        cols.append(node + off)
        vals.append(np.full(n, diag_value if off == 0 else off_value, dtype=np.float32))
        valid.append(mask)
    cols = np.stack(cols, axis=1)
    vals = np.stack(vals, axis=1)
    valid = np.stack(valid, axis=1)
    counts = valid.sum(axis=1)
    indptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(counts, out=indptr[1:])
    return (vals[valid].astype(np.float32), cols[valid].astype(index_dtype), indptr.astype(index_dtype))


def lap2d(m: int, index_dtype=np.int32):
    n = m * m
    node = np.arange(n, dtype=np.int64)
    i, j = node // m, node % m
    stencil = [(-m, i > 0), (-1, j > 0), (0, np.ones(n, bool)), (1, j < m - 1), (m, i < m - 1)]
    return _stencil_csr(n, stencil, 4.0, -1.0, index_dtype), (n, n)


def poisson3d(m: int, index_dtype=np.int32):
    n = m * m * m
    node = np.arange(n, dtype=np.int64)
    i, j, k = node // (m * m), (node // m) % m, node % m
    mm = m * m
    stencil = [(-mm, i > 0), (-m, j > 0), (-1, k > 0), (0, np.ones(n, bool)), (1, k < m - 1), (m, j < m - 1),
               (mm, i < m - 1)]
    return _stencil_csr(n, stencil, 6.0, -1.0, index_dtype), (n, n)


def _distinct_sorted_columns(rng, row_of: np.ndarray, n_cols: int) -> np.ndarray:
    """Uniform columns, distinct within each row, sorted; rows given per entry."""
    cols = rng.integers(0, n_cols, size=row_of.shape[0], dtype=np.int64)
    while True:
        key = row_of * n_cols + cols
        order = np.argsort(key, kind="stable")
        key = key[order]
        dup = np.zeros(key.shape[0], dtype=bool)
        dup[1:] = key[1:] == key[:-1]
        cols = cols[order]
        row_of = row_of[order]
        n_dup = int(dup.sum())
        if n_dup == 0:
            return cols
        cols[dup] = rng.integers(0, n_cols, size=n_dup, dtype=np.int64)


def random_k_per_row(n_rows: int, n_cols: int, k: int, seed: int, index_dtype=np.int32):
    rng = np.random.default_rng(seed)
    row_of = np.repeat(np.arange(n_rows, dtype=np.int64), k)
    cols = _distinct_sorted_columns(rng, row_of, n_cols)
    data = rng.standard_normal(cols.shape[0]).astype(np.float32)
    indptr = np.arange(0, n_rows * k + 1, k, dtype=np.int64)
    return (data, cols.astype(index_dtype), indptr.astype(index_dtype)), (n_rows, n_cols)


POWER_LAW_ALPHA = 2.1
POWER_LAW_CAP = 65536
POWER_LAW_SCALE = 21.5


def power_law_lengths(n: int, rng, alpha=POWER_LAW_ALPHA, scale=POWER_LAW_SCALE, cap=POWER_LAW_CAP):
    """Discrete Lomax lengths: 1 + floor(scale * ((1-U)^(-1/alpha) - 1)), capped."""
    u = rng.random(n)
    lengths = 1 + np.floor(scale * ((1.0 - u) ** (-1.0 / alpha) - 1.0))
    return np.minimum(lengths, cap).astype(np.int64)


def power_law(n: int, seed: int, index_dtype=np.int64):
    rng = np.random.default_rng(seed)
    lengths = power_law_lengths(n, rng)
    lengths = np.minimum(lengths, n)
    indptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(lengths, out=indptr[1:])
    row_of = np.repeat(np.arange(n, dtype=np.int64), lengths)
    cols = _distinct_sorted_columns(rng, row_of, n)
    data = rng.uniform(-1.0, 1.0, cols.shape[0]).astype(np.float32)
    return (data, cols.astype(index_dtype), indptr.astype(index_dtype)), (n, n)


def uniform_vector(n: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).uniform(-1.0, 1.0, n).astype(np.float32)


def uniform_matrix(rows: int, cols: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).uniform(-1.0, 1.0, (rows, cols)).astype(np.float32)


def random_csr(n_rows: int, n_cols: int, density: float, seed: int, index_dtype=np.int32, dtype=np.float32):
    """scipy.sparse.random-like canonical CSR (values N(0,1))."""
    rng = np.random.default_rng(seed)
    nnz_target = int(round(density * n_rows * n_cols))
    flat = rng.choice(n_rows * n_cols, size=nnz_target, replace=False) if nnz_target else np.zeros(0, np.int64)
    flat = np.sort(flat)
    rows, cols = flat // n_cols, flat % n_cols
    data = rng.standard_normal(flat.shape[0]).astype(dtype)
    indptr = np.zeros(n_rows + 1, dtype=np.int64)
    np.add.at(indptr, rows + 1, 1)
    np.cumsum(indptr, out=indptr)
    return (data, cols.astype(index_dtype), indptr.astype(index_dtype)), (n_rows, n_cols)


def ragged_csr(n_rows: int, n_cols: int, seed: int, max_len: int, index_dtype=np.int32, empty_frac=0.2):
    """Rows of very different lengths (including empty and a few long ones)."""
    rng = np.random.default_rng(seed)
    lengths = rng.integers(0, max_len + 1, size=n_rows)
    lengths[rng.random(n_rows) < empty_frac] = 0
    if n_rows >= 4:
        lengths[rng.integers(0, n_rows, size=2)] = min(n_cols, max_len * 40)
    lengths = np.minimum(lengths, n_cols)
    indptr = np.zeros(n_rows + 1, dtype=np.int64)
    np.cumsum(lengths, out=indptr[1:])
    row_of = np.repeat(np.arange(n_rows, dtype=np.int64), lengths)
    cols = _distinct_sorted_columns(rng, row_of, n_cols)
    data = rng.uniform(-1.0, 1.0, cols.shape[0]).astype(np.float32)
    return (data, cols.astype(index_dtype), indptr.astype(index_dtype)), (n_rows, n_cols)
