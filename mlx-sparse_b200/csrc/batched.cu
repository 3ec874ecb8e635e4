// Batched products: one CSR matrix times a batch of dense vectors or matrices.
//
// Reference behaviour: csr_batched_matvec_cpu_impl
// (src/sparse/csr_batched_matvec/csr_batched_matvec.cpp:82-130) computes, for
// every (batch b, row r), acc = sum over the row's nonzeros, in order, of
// a * x[b, col] with the fp32 accumulator of the value type, then casts;
// csr_batched_matmul (src/sparse/csr_batched_matmul/csr_batched_matmul.cpp)
// does the same per output column of every batch.
//
// B200 design. A batch of vectors is one SpMM: X [batch, n_cols] is
// transposed (tiled through shared memory) into X^T [n_cols, batch], so every
// nonzero gathers `batch` contiguous values instead of `batch` scattered ones;
// the SpMM kernel sums each output element over the row's nonzeros in order
// (bit-identical to the reference's per-element loop), and the [n_rows, batch]
// result is transposed back. A batch of matrices runs the SpMM kernel once per
// batch entry on the caller's stream (each entry is already a row-major
// [n_cols, k] block).
#include "ops.cuh"

namespace msx {

namespace {

constexpr int kTile = 32;

// out[c * rows + r] = in[r * cols + c]; one 32x32 tile per CTA (1D grid of
// tiles, column tiles fastest), 32x8 threads.
template <typename T>
__global__ void __launch_bounds__(kTile * 8)
transpose_kernel(const T *__restrict__ in, T *__restrict__ out, int64_t rows, int64_t cols, int64_t tiles_x) {
  __shared__ T tile[kTile][kTile + 1];
  const int64_t t = blockIdx.x;
  const int64_t r0 = (t / tiles_x) * kTile, c0 = (t % tiles_x) * kTile;
  for (int i = threadIdx.y; i < kTile; i += 8) {
    const int64_t r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = in[r * cols + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < kTile; i += 8) {
    const int64_t c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[c * rows + r] = tile[threadIdx.x][i];
  }
}

void transpose(int value_dtype, const void *in, void *out, int64_t rows, int64_t cols, cudaStream_t s) {
  if (rows == 0 || cols == 0) return;
  const int64_t tiles_x = ceil_div(cols, kTile), tiles = tiles_x * ceil_div(rows, kTile);
  if (tiles > INT32_MAX) fail(MSX_ERR_OVERFLOW, "batched product: operand too large for one transpose launch.");
  dim3 grid((unsigned)tiles), block(kTile, 8);
  dispatch_value(value_dtype, [&](auto vt) {
    using T = decltype(vt);
    transpose_kernel<T><<<grid, block, 0, s>>>(static_cast<const T *>(in), static_cast<T *>(out), rows, cols,
                                               tiles_x);
  });
  MSX_CHECK_LAUNCH();
}

}  // namespace

void csr_batched_matvec_run(int value_dtype, int index_dtype, const void *data, const void *indices,
                            const void *indptr, int64_t nnz, int64_t n_rows, int64_t n_cols, int64_t batch,
                            const void *rhs, void *out, cudaStream_t s) {
  if (batch == 0 || n_rows == 0) return;
  const size_t elem = value_dtype == MSX_F32 ? 4 : 2;
  if (batch == 1) {  // X^T is X itself
    spmm_run(value_dtype, index_dtype, data, indices, indptr, rhs, 1, out, n_rows, n_cols, nnz, s);
    return;
  }
  Scratch xt(elem * (size_t)(n_cols * batch), s);
  Scratch yt(elem * (size_t)(n_rows * batch), s);
  transpose(value_dtype, rhs, xt.ptr, batch, n_cols, s);
  spmm_run(value_dtype, index_dtype, data, indices, indptr, xt.ptr, batch, yt.ptr, n_rows, n_cols, nnz, s);
  transpose(value_dtype, yt.ptr, out, n_rows, batch, s);
}

void csr_batched_matmul_run(int value_dtype, int index_dtype, const void *data, const void *indices,
                            const void *indptr, int64_t nnz, int64_t n_rows, int64_t n_cols, int64_t batch,
                            int64_t k, const void *rhs, void *out, cudaStream_t s) {
  if (batch == 0 || n_rows == 0 || k == 0) return;
  const size_t elem = value_dtype == MSX_F32 ? 4 : 2;
  const char *b = static_cast<const char *>(rhs);
  char *o = static_cast<char *>(out);
  for (int64_t i = 0; i < batch; ++i)
    spmm_run(value_dtype, index_dtype, data, indices, indptr, b + elem * (size_t)(i * n_cols * k), k,
             o + elem * (size_t)(i * n_rows * k), n_rows, n_cols, nnz, s);
}

}  // namespace msx
