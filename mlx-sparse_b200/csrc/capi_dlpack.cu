// DLPack form of the C ABI (include/msx_sparse.h, "DLPack entry points").
//
// The reference's Python layer hands device arrays to its native module
// (mlx_sparse/_native.py:179-189 -> src/bindings.cpp:874-1161); here every
// array crosses as a DLTensor. Each wrapper checks the tensors (CUDA device =
// the current device, dtype, rank, shape, compact strides), resolves
// data + byte_offset and calls the raw-pointer entry point, so both forms run
// the same kernels.
#include <string>

#include "common.cuh"

namespace msx {

void require(bool ok, int status, const std::string &msg);

namespace {

constexpr int32_t kDLCUDA = 2, kDLCUDAManaged = 13;
constexpr uint8_t kDLInt = 0, kDLFloat = 2, kDLBfloat = 4;

struct View {
  void *ptr = nullptr;
  int64_t numel = 0;
  int64_t dim0 = 0, dim1 = 1;
};

// Checks device, rank and compactness; returns the element pointer.
View view(const DLTensor *t, const char *op, const char *name, int min_rank, int max_rank) {
  const std::string what = std::string(op) + " " + name;
  if (t == nullptr) fail(MSX_ERR_INVALID, what + " must not be null.");
  if (t->device.device_type != kDLCUDA && t->device.device_type != kDLCUDAManaged)
    fail(MSX_ERR_INVALID, what + " must be a CUDA device tensor (DLPack device type " +
                              std::to_string(t->device.device_type) + "); there is no CPU fallback.");
  int cur = 0;
  MSX_CUDA(cudaGetDevice(&cur));
  if (t->device.device_id != cur)
    fail(MSX_ERR_INVALID, what + " lives on device " + std::to_string(t->device.device_id) +
                              " but the current device is " + std::to_string(cur) + ".");
  if (t->ndim < min_rank || t->ndim > max_rank)
    fail(MSX_ERR_INVALID, what + " must be rank-" + std::to_string(min_rank) +
                              (max_rank > min_rank ? " or rank-" + std::to_string(max_rank) : "") + ", got rank-" +
                              std::to_string(t->ndim) + ".");
  if (t->dtype.lanes != 1) fail(MSX_ERR_TYPE, what + " must have one lane per element.");
  View v;
  v.numel = 1;
  for (int d = 0; d < t->ndim; ++d) {
    if (t->shape[d] < 0) fail(MSX_ERR_INVALID, what + " has a negative dimension.");
    v.numel *= t->shape[d];
  }
  if (t->strides && v.numel > 0) {
    int64_t expect = 1;
    for (int d = t->ndim - 1; d >= 0; --d) {
      if (t->shape[d] != 1 && t->strides[d] != expect)
        fail(MSX_ERR_INVALID, what + " must be contiguous (compact row-major strides).");
      expect *= t->shape[d];
    }
  }
  v.dim0 = t->ndim >= 1 ? t->shape[0] : 1;
  v.dim1 = t->ndim >= 2 ? t->shape[1] : 1;
  v.ptr = static_cast<char *>(t->data) + t->byte_offset;
  return v;
}

int value_code(const DLTensor *t, const char *op, const char *name) {
  const DLDataType d = t->dtype;
  if (d.code == kDLFloat && d.bits == 32) return MSX_F32;
  if (d.code == kDLFloat && d.bits == 16) return MSX_F16;
  if (d.code == kDLBfloat && d.bits == 16) return MSX_BF16;
  fail(MSX_ERR_TYPE, std::string(op) + " " + name + " dtype must be one of float32, float16, bfloat16.");
}

int index_code(const DLTensor *t, const char *op, const char *name) {
  const DLDataType d = t->dtype;
  if (d.code == kDLInt && d.bits == 32) return MSX_I32;
  if (d.code == kDLInt && d.bits == 64) return MSX_I64;
  fail(MSX_ERR_TYPE, std::string(op) + " " + name + " dtype must be one of int32, int64.");
}

struct Csr {
  View data, indices, indptr;
  int vt, it;
};

// A CSR triple: matching lengths, one index dtype, indptr of n_rows + 1.
Csr csr(const DLTensor *data, const DLTensor *indices, const DLTensor *indptr, int64_t n_rows, const char *op) {
  Csr c;
  c.data = view(data, op, "data", 1, 1);
  c.indices = view(indices, op, "indices", 1, 1);
  c.indptr = view(indptr, op, "indptr", 1, 1);
  c.vt = value_code(data, op, "data");
  c.it = index_code(indices, op, "indices");
  if (index_code(indptr, op, "indptr") != c.it)
    fail(MSX_ERR_TYPE, std::string(op) + " indices and indptr must share an index dtype.");
  require(c.data.numel == c.indices.numel, MSX_ERR_INVALID,
          std::string(op) + " data and indices must have equal length.");
  require(c.indptr.numel == n_rows + 1, MSX_ERR_INVALID,
          std::string(op) + " indptr must have length n_rows + 1 = " + std::to_string(n_rows + 1) + ".");
  return c;
}

void same_value_dtype(const DLTensor *t, int vt, const char *op, const char *name) {
  if (value_code(t, op, name) != vt)
    fail(MSX_ERR_TYPE, std::string(op) + " " + name + " must have the sparse data's dtype.");
}

void float32(const DLTensor *t, const char *op, const char *name) {
  if (value_code(t, op, name) != MSX_F32)
    fail(MSX_ERR_TYPE, std::string(op) + " " + name + " currently requires dtype float32.");
}

// Runs `fn` (a raw entry point call) inside the DLPack wrapper's guard: the
// raw call has already set the thread's message, so its status is rethrown.
template <typename Fn> void forward(Fn &&fn) {
  const int rc = fn();
  if (rc != MSX_OK) throw Error(rc, msx_last_error());
}

}  // namespace
}  // namespace msx

using namespace msx;

extern "C" {

int msx_dl_csr_matvec(const DLTensor *data, const DLTensor *indices, const DLTensor *indptr, const DLTensor *x,
                      DLTensor *y, int64_t n_rows, int64_t n_cols, const msx_spmv_plan *plan, void *stream) {
  return guarded([&] {
    const char *op = "csr_matvec";
    require(n_rows >= 0 && n_cols >= 0, MSX_ERR_INVALID, "csr_matvec shape dimensions must be non-negative.");
    Csr a = csr(data, indices, indptr, n_rows, op);
    View xv = view(x, op, "x", 1, 1), yv = view(y, op, "y", 1, 1);
    same_value_dtype(x, a.vt, op, "x");
    same_value_dtype(y, a.vt, op, "y");
    require(xv.numel == n_cols, MSX_ERR_INVALID, "csr_matvec x must have length n_cols.");
    require(yv.numel == n_rows, MSX_ERR_INVALID, "csr_matvec y must have length n_rows.");
    forward([&] {
      return msx_csr_matvec(a.vt, a.it, a.data.ptr, a.indices.ptr, a.indptr.ptr, a.data.numel, xv.ptr, yv.ptr, n_rows,
                            n_cols, plan, stream);
    });
  });
}

int msx_dl_csr_matmul(const DLTensor *data, const DLTensor *indices, const DLTensor *indptr, const DLTensor *rhs,
                      DLTensor *out, int64_t n_rows, int64_t n_cols, void *stream) {
  return guarded([&] {
    const char *op = "csr_matmul";
    require(n_rows >= 0 && n_cols >= 0, MSX_ERR_INVALID, "csr_matmul shape dimensions must be non-negative.");
    Csr a = csr(data, indices, indptr, n_rows, op);
    View bv = view(rhs, op, "rhs", 2, 2), ov = view(out, op, "out", 2, 2);
    same_value_dtype(rhs, a.vt, op, "rhs");
    same_value_dtype(out, a.vt, op, "out");
    require(bv.dim0 == n_cols, MSX_ERR_INVALID,
            "csr_matmul rhs first dimension must equal the sparse matrix column count.");
    require(ov.dim0 == n_rows && ov.dim1 == bv.dim1, MSX_ERR_INVALID, "csr_matmul out must have shape (n_rows, k).");
    forward([&] {
      return msx_csr_matmul(a.vt, a.it, a.data.ptr, a.indices.ptr, a.indptr.ptr, a.data.numel, bv.ptr, bv.dim1, ov.ptr,
                            n_rows, n_cols, stream);
    });
  });
}

int msx_dl_csr_matmat_symbolic(const DLTensor *lhs_data, const DLTensor *lhs_indices, const DLTensor *lhs_indptr,
                               const DLTensor *rhs_data, const DLTensor *rhs_indices, const DLTensor *rhs_indptr,
                               int64_t lhs_n_rows, int64_t lhs_n_cols, int64_t rhs_n_rows, int64_t rhs_n_cols,
                               DLTensor *out_indptr, int64_t *out_nnz, int prune_zeros, void *stream) {
  return guarded([&] {
    const char *op = "csr_matmat";
    Csr l = csr(lhs_data, lhs_indices, lhs_indptr, lhs_n_rows, op);
    Csr r = csr(rhs_data, rhs_indices, rhs_indptr, rhs_n_rows, op);
    if (l.vt != r.vt) fail(MSX_ERR_TYPE, "CSR sparse-sparse matmul requires matching value dtypes.");
    View pv = view(out_indptr, op, "out_indptr", 1, 1);
    const int out_it = l.it == r.it ? l.it : MSX_I64;
    if (index_code(out_indptr, op, "out_indptr") != out_it)
      fail(MSX_ERR_TYPE, "csr_matmat out_indptr must use the output index dtype (int64 unless both are int32).");
    require(pv.numel == lhs_n_rows + 1, MSX_ERR_INVALID, "csr_matmat out_indptr must have length lhs_n_rows + 1.");
    forward([&] {
      return msx_csr_matmat_symbolic(l.vt, l.it, l.data.ptr, l.indices.ptr, l.indptr.ptr, l.data.numel, r.it,
                                     r.data.ptr, r.indices.ptr, r.indptr.ptr, r.data.numel, lhs_n_rows, lhs_n_cols,
                                     rhs_n_rows, rhs_n_cols, out_it, pv.ptr, out_nnz, prune_zeros, stream);
    });
  });
}

int msx_dl_csr_matmat_numeric(const DLTensor *lhs_data, const DLTensor *lhs_indices, const DLTensor *lhs_indptr,
                              const DLTensor *rhs_data, const DLTensor *rhs_indices, const DLTensor *rhs_indptr,
                              int64_t lhs_n_rows, int64_t lhs_n_cols, int64_t rhs_n_rows, int64_t rhs_n_cols,
                              const DLTensor *out_indptr, DLTensor *out_data, DLTensor *out_indices, int prune_zeros,
                              void *stream) {
  return guarded([&] {
    const char *op = "csr_matmat";
    Csr l = csr(lhs_data, lhs_indices, lhs_indptr, lhs_n_rows, op);
    Csr r = csr(rhs_data, rhs_indices, rhs_indptr, rhs_n_rows, op);
    if (l.vt != r.vt) fail(MSX_ERR_TYPE, "CSR sparse-sparse matmul requires matching value dtypes.");
    const int out_it = l.it == r.it ? l.it : MSX_I64;
    View pv = view(out_indptr, op, "out_indptr", 1, 1);
    View dv = view(out_data, op, "out_data", 1, 1), iv = view(out_indices, op, "out_indices", 1, 1);
    if (index_code(out_indptr, op, "out_indptr") != out_it || index_code(out_indices, op, "out_indices") != out_it)
      fail(MSX_ERR_TYPE, "csr_matmat outputs must use the output index dtype (int64 unless both are int32).");
    same_value_dtype(out_data, l.vt, op, "out_data");
    require(dv.numel == iv.numel, MSX_ERR_INVALID, "csr_matmat out_data and out_indices must have equal length.");
    forward([&] {
      return msx_csr_matmat_numeric(l.vt, l.it, l.data.ptr, l.indices.ptr, l.indptr.ptr, l.data.numel, r.it,
                                    r.data.ptr, r.indices.ptr, r.indptr.ptr, r.data.numel, lhs_n_rows, lhs_n_cols,
                                    rhs_n_rows, rhs_n_cols, out_it, pv.ptr, dv.numel, dv.ptr, iv.ptr, prune_zeros,
                                    stream);
    });
  });
}

static void solver_views(const char *op, const DLTensor *data, const DLTensor *indices, const DLTensor *indptr,
                         const DLTensor *b, const DLTensor *x0, const DLTensor *x_out, int64_t n_rows,
                         int64_t n_cols, Csr &a, View &bv, View &x0v, View &xv) {
  a = csr(data, indices, indptr, n_rows, op);
  float32(data, op, "data");
  bv = view(b, op, "b", 1, 1);
  x0v = view(x0, op, "x0", 1, 1);
  xv = view(x_out, op, "x", 1, 1);
  float32(b, op, "b");
  float32(x0, op, "x0");
  float32(x_out, op, "x");
  require(bv.numel == n_rows, MSX_ERR_INVALID, std::string(op) + " b must have length n_rows.");
  require(x0v.numel == n_cols && xv.numel == n_rows, MSX_ERR_INVALID,
          std::string(op) + " x0 must have length n_cols and x length n_rows.");
}

int msx_dl_csr_cg(const DLTensor *data, const DLTensor *indices, const DLTensor *indptr, const DLTensor *b,
                  const DLTensor *x0, DLTensor *x_out, int64_t n_rows, int64_t n_cols, float rtol, float atol,
                  int32_t maxiter, int32_t *info, float *residual, int32_t *iterations, void *stream) {
  return guarded([&] {
    Csr a;
    View bv, x0v, xv;
    solver_views("csr_cg", data, indices, indptr, b, x0, x_out, n_rows, n_cols, a, bv, x0v, xv);
    forward([&] {
      return msx_csr_cg(a.it, static_cast<const float *>(a.data.ptr), a.indices.ptr, a.indptr.ptr, a.data.numel,
                        static_cast<const float *>(bv.ptr), static_cast<const float *>(x0v.ptr),
                        static_cast<float *>(xv.ptr), n_rows, n_cols, rtol, atol, maxiter, info, residual, iterations,
                        stream);
    });
  });
}

int msx_dl_csr_pcg_jacobi(const DLTensor *data, const DLTensor *indices, const DLTensor *indptr, const DLTensor *b,
                          const DLTensor *x0, const DLTensor *inv_diag, DLTensor *x_out, int64_t n_rows,
                          int64_t n_cols, float rtol, float atol, int32_t maxiter, int32_t *info, float *residual,
                          int32_t *iterations, void *stream) {
  return guarded([&] {
    const char *op = "csr_pcg_jacobi";
    Csr a;
    View bv, x0v, xv;
    solver_views(op, data, indices, indptr, b, x0, x_out, n_rows, n_cols, a, bv, x0v, xv);
    View iv = view(inv_diag, op, "inv_diag", 1, 1);
    float32(inv_diag, op, "inv_diag");
    require(iv.numel == n_rows, MSX_ERR_INVALID, "csr_pcg_jacobi inv_diag must have length n_rows.");
    forward([&] {
      return msx_csr_pcg_jacobi(a.it, static_cast<const float *>(a.data.ptr), a.indices.ptr, a.indptr.ptr,
                                a.data.numel, static_cast<const float *>(bv.ptr), static_cast<const float *>(x0v.ptr),
                                static_cast<const float *>(iv.ptr), static_cast<float *>(xv.ptr), n_rows, n_cols,
                                rtol, atol, maxiter, info, residual, iterations, stream);
    });
  });
}

}  // extern "C"
