// Host-side entry points of the kernel families, called by capi.cu.
#pragma once
#include "common.cuh"

namespace msx {

void spmm_run(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
              const void *rhs, int64_t k, void *out, int64_t n_rows, int64_t n_cols, int64_t nnz,
              cudaStream_t stream);

void spgemm_run(bool write, int value_dtype, int lhs_it, const void *ld, const void *li, const void *lp, int rhs_it,
                const void *rd, const void *ri, const void *rp, int64_t m, int64_t rhs_rows, int64_t n_cols,
                int out_it, void *out_indptr, void *out_idx, void *out_data, int64_t *out_nnz, bool prune,
                cudaStream_t s);

void csr_batched_matvec_run(int value_dtype, int index_dtype, const void *data, const void *indices,
                            const void *indptr, int64_t nnz, int64_t n_rows, int64_t n_cols, int64_t batch,
                            const void *rhs, void *out, cudaStream_t s);
void csr_batched_matmul_run(int value_dtype, int index_dtype, const void *data, const void *indices,
                            const void *indptr, int64_t nnz, int64_t n_rows, int64_t n_cols, int64_t batch,
                            int64_t k, const void *rhs, void *out, cudaStream_t s);

void csr_diagonal_run(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
                      int64_t n_diag, void *out, cudaStream_t stream);

// COO -> CSR (by_col: rows sorted by (column, source position) as the
// reference's coo_tocsr; else by source position only). out_data may be null
// (structure only); out_perm (int64[nnz], the source position of every output
// entry) may be null. Synchronises `s` once (coordinate check).
void coo_tocsr_run(int value_dtype, int index_dtype, const void *data, const void *row, const void *col, int64_t nnz,
                   int64_t n_rows, int64_t n_cols, bool by_col, void *out_data, void *out_indices, void *out_indptr,
                   int64_t *out_perm, cudaStream_t s);
// CSR of A^T: row c lists A's entries of column c by ascending row.
void csr_transpose_run(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
                       int64_t nnz, int64_t n_rows, int64_t n_cols, void *out_data, void *out_indices,
                       void *out_indptr, int64_t *out_perm, cudaStream_t s);
// out[p] = sum_j cot[row(p), j] * rhs[col(p), j], j in order (k = 1: matvec).
void csr_data_vjp_run(int value_dtype, int index_dtype, const void *indices, const void *indptr, int64_t nnz,
                      int64_t n_rows, const void *rhs, const void *cot, int64_t k, void *out, cudaStream_t s);

}  // namespace msx
