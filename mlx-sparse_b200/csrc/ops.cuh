// Host-side entry points of the kernel families, called by capi.cu.
#pragma once
#include "common.cuh"

namespace msx {

void spmm_run(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
              const void *rhs, int64_t k, void *out, int64_t n_rows, int64_t n_cols, cudaStream_t stream);

}  // namespace msx
