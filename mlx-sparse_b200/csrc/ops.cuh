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

}  // namespace msx
