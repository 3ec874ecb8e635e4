// C-ABI entry points (include/msx_sparse.h). Argument checks follow the
// reference front-ends (e.g. src/sparse/csr_matvec/csr_matvec.cpp:326-356) and
// map C++ exception kinds onto msx_status codes.
#include <cmath>
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>
#if defined(MSX_HAVE_NCCL)
#include <nccl.h>
#endif
#include <string>

#include "msx_sparse.h"
#include "cg.cuh"
#include "ops.cuh"
#include "spmv.cuh"
#include "spmv_binned.cuh"

namespace msx {

static thread_local std::string g_last_error;
void set_last_error(const std::string &msg) { g_last_error = msg; }

void require(bool ok, int status, const std::string &msg) {
  if (!ok) fail(status, msg);
}

void check_ptr(const void *p, int64_t count, const char *name) {
  if (count > 0 && p == nullptr) fail(MSX_ERR_INVALID, std::string(name) + " must not be null.");
}

}  // namespace msx

struct msx_spmv_plan {
  void *dev = nullptr;  // one cudaMalloc holding the binned plan's arrays
  void *tiles = nullptr;  // merge-path tile boundaries
  int device = 0;
  int64_t n_tiles = 0, n_split = 0;
  bool use_tiles = false;
  msx::BinnedPlan bins;
};

namespace {
// Kernel used by planned products: row-length bins when every row falls in
// one bin (stencils: the short-row kernels stage each block's contiguous
// nonzeros), else merge-path tiles, which read the matrix in row order (on a
// 2^22-row power-law matrix 0.551 ms against 0.588 for the bins, whose
// permuted rows re-fetch shared sectors). MSX_SPMV_KERNEL=tiles / bins forces
// either.
int planned_kernel_override() {
  static const int v = [] {
    const char *e = getenv("MSX_SPMV_KERNEL");
    if (e && std::string(e) == "tiles") return 1;
    if (e && std::string(e) == "bins") return 2;
    return 0;
  }();
  return v;
}
}  // namespace

// A persistent CG solver (one matrix, one rank) with copies of its peer lists.
struct msx_cg_context {
  msx::CgEngine *engine = nullptr;
  std::vector<int> peers;
  std::vector<int64_t> send_counts, recv_counts, dst_offset;
  int world = 1;
  ~msx_cg_context() { msx::cg_engine_destroy(engine); }
};

using namespace msx;

extern "C" {

const char *msx_last_error(void) { return g_last_error.c_str(); }

int msx_version(void) { return 1; }

int msx_compiled_sm(void) {
#if defined(MSX_SM)
  return MSX_SM;
#else
  return 0;
#endif
}

int msx_check_device_errors(void *stream) {
  return guarded([&] {
    MSX_CUDA(cudaStreamSynchronize(as_stream(stream)));
    if (spmv_take_error())
      fail(MSX_ERR_RUNTIME,
           "an SpMV bulk-copy wait on this device gave up (poll limit reached); the results of SpMV calls "
           "made since the last check are incomplete.");
  });
}

int msx_debug_set_spmv_poll_limit(int64_t polls) {
  return guarded([&] { spmv_set_poll_limit(polls); });
}

int msx_spmv_plan_create(int index_dtype, const void *indptr, int64_t n_rows, int64_t nnz, void *stream,
                         msx_spmv_plan **out) {
  return guarded([&] {
    require(out != nullptr, MSX_ERR_INVALID, "msx_spmv_plan_create: out must not be null.");
    *out = nullptr;
    require(n_rows >= 0 && nnz >= 0, MSX_ERR_INVALID, "csr_matvec shape dimensions must be non-negative.");
    check_ptr(indptr, n_rows + 1, "csr_matvec indptr");
    dispatch_index(index_dtype, [](auto) {});
    auto *plan = new msx_spmv_plan();
    MSX_CUDA(cudaGetDevice(&plan->device));
    try {
      auto alloc = [&](size_t bytes) -> void * {
        cudaError_t e = cudaMalloc(&plan->dev, bytes);
        if (e != cudaSuccess)
          fail(MSX_ERR_CUDA, std::string("cudaMalloc for the SpMV plan failed: ") + cudaGetErrorString(e));
        return plan->dev;
      };
      build_binned_plan(index_dtype, indptr, n_rows, nnz, as_stream(stream), alloc, plan->bins);
      const int force = planned_kernel_override();
      plan->use_tiles = force == 1 || (force == 0 && !plan->bins.info.identity);
      plan->n_tiles = spmv_num_tiles(n_rows, nnz);
      cudaError_t e = cudaMalloc(&plan->tiles, spmv_plan_device_bytes(plan->n_tiles));
      if (e != cudaSuccess)
        fail(MSX_ERR_CUDA, std::string("cudaMalloc for the SpMV plan failed: ") + cudaGetErrorString(e));
      cudaStream_t s = as_stream(stream);
      spmv_build_plan(index_dtype, indptr, n_rows, nnz, plan->tiles, plan->n_tiles, s);
      int64_t *tr, *tn;
      unsigned long long *ns, split = 0;
      spmv_plan_layout(plan->tiles, plan->n_tiles, &tr, &tn, &ns);
      MSX_CUDA(cudaMemcpyAsync(&split, ns, sizeof(split), cudaMemcpyDeviceToHost, s));
      MSX_CUDA(cudaStreamSynchronize(s));
      plan->n_split = (int64_t)split;
    } catch (...) {
      if (plan->dev) cudaFree(plan->dev);
      if (plan->tiles) cudaFree(plan->tiles);
      delete plan;
      throw;
    }
    *out = plan;
  });
}

int msx_spmv_plan_destroy(msx_spmv_plan *plan) {
  return guarded([&] {
    if (!plan) return;
    if (plan->dev || plan->tiles) {
      int cur = 0;
      cudaGetDevice(&cur);
      if (cur != plan->device) cudaSetDevice(plan->device);
      if (plan->dev) cudaFree(plan->dev);
      if (plan->tiles) cudaFree(plan->tiles);
      if (cur != plan->device) cudaSetDevice(cur);
    }
    delete plan;
  });
}

int msx_spmv_plan_info(const msx_spmv_plan *plan, int64_t *n_blocks, int64_t *n_long_rows) {
  return guarded([&] {
    require(plan != nullptr, MSX_ERR_INVALID, "plan must not be null.");
    if (n_blocks) *n_blocks = plan->use_tiles ? plan->n_tiles : binned_blocks(plan->bins);
    if (n_long_rows) *n_long_rows = plan->use_tiles ? plan->n_split : plan->bins.n_long;
  });
}

int msx_csr_matvec(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
                   int64_t nnz, const void *x, void *y, int64_t n_rows, int64_t n_cols, const msx_spmv_plan *plan,
                   void *stream) {
  return guarded([&] {
    require(n_rows >= 0 && n_cols >= 0, MSX_ERR_INVALID, "csr_matvec shape dimensions must be non-negative.");
    require(nnz >= 0, MSX_ERR_INVALID, "csr_matvec nnz must be non-negative.");
    dispatch_value(value_dtype, [](auto) {});
    dispatch_index(index_dtype, [](auto) {});
    check_ptr(data, nnz, "csr_matvec data");
    check_ptr(indices, nnz, "csr_matvec indices");
    check_ptr(indptr, n_rows + 1, "csr_matvec indptr");
    check_ptr(x, nnz > 0 ? n_cols : 0, "csr_matvec x");
    check_ptr(y, n_rows, "csr_matvec y");
    if (n_rows == 0) return;
    cudaStream_t s = as_stream(stream);
    if (plan) {
      require(plan->bins.n_rows == n_rows && plan->bins.nnz == nnz, MSX_ERR_INVALID,
              "csr_matvec plan was built for a different matrix shape.");
      if (plan->use_tiles) {
        Scratch carry(plan->n_split > 0 ? sizeof(float) * 2 * plan->n_tiles : 0, s);
        spmv_run(value_dtype, index_dtype, data, indices, indptr, x, y, n_rows, nnz, plan->tiles, plan->n_tiles,
                 plan->n_split > 0, carry.as<float>(), s);
        return;
      }
      Scratch carry(sizeof(float) * plan->bins.n_chunks, s);
      spmv_binned_run(value_dtype, index_dtype, plan->bins, data, indices, indptr, x, y, carry.as<float>(), s);
      return;
    }
    const int64_t n_tiles = spmv_num_tiles(n_rows, nnz);
    const size_t plan_bytes = spmv_plan_device_bytes(n_tiles);
    Scratch scratch(plan_bytes + sizeof(float) * 2 * n_tiles, s);
    char *base = scratch.as<char>();
    spmv_build_plan(index_dtype, indptr, n_rows, nnz, base, n_tiles, s);
    spmv_run(value_dtype, index_dtype, data, indices, indptr, x, y, n_rows, nnz, base, n_tiles, true,
             reinterpret_cast<float *>(base + plan_bytes), s);
  });
}

int msx_csr_matmul(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
                   int64_t nnz, const void *rhs, int64_t rhs_cols, void *out, int64_t n_rows, int64_t n_cols,
                   void *stream) {
  return guarded([&] {
    require(n_rows >= 0 && n_cols >= 0, MSX_ERR_INVALID, "csr_matmul shape dimensions must be non-negative.");
    require(nnz >= 0 && rhs_cols >= 0, MSX_ERR_INVALID, "csr_matmul sizes must be non-negative.");
    dispatch_value(value_dtype, [](auto) {});
    dispatch_index(index_dtype, [](auto) {});
    check_ptr(data, nnz, "csr_matmul data");
    check_ptr(indices, nnz, "csr_matmul indices");
    check_ptr(indptr, n_rows + 1, "csr_matmul indptr");
    check_ptr(rhs, nnz > 0 ? n_cols * rhs_cols : 0, "csr_matmul rhs");
    check_ptr(out, n_rows * rhs_cols, "csr_matmul out");
    spmm_run(value_dtype, index_dtype, data, indices, indptr, rhs, rhs_cols, out, n_rows, n_cols, nnz,
             as_stream(stream));
  });
}

int msx_coo_tocsr(int value_dtype, int index_dtype, const void *data, const void *row, const void *col, int64_t nnz,
                  int64_t n_rows, int64_t n_cols, int sort_columns, void *out_data, void *out_indices,
                  void *out_indptr, int64_t *out_perm, void *stream) {
  return guarded([&] {
    require(n_rows >= 0 && n_cols >= 0, MSX_ERR_INVALID, "coo_tocsr shape dimensions must be non-negative.");
    require(nnz >= 0, MSX_ERR_INVALID, "coo_tocsr nnz must be non-negative.");
    dispatch_value(value_dtype, [](auto) {});
    dispatch_index(index_dtype, [](auto) {});
    if (index_dtype == MSX_I32 && nnz > INT32_MAX)
      fail(MSX_ERR_OVERFLOW, "coo_tocsr nnz exceeds the int32 index capacity.");
    check_ptr(row, nnz, "coo_tocsr row");
    check_ptr(col, nnz, "coo_tocsr col");
    check_ptr(out_indices, nnz, "coo_tocsr out_indices");
    check_ptr(out_indptr, n_rows + 1, "coo_tocsr out_indptr");
    if (out_data) check_ptr(data, nnz, "coo_tocsr data");
    coo_tocsr_run(value_dtype, index_dtype, data, row, col, nnz, n_rows, n_cols, sort_columns != 0, out_data,
                  out_indices, out_indptr, out_perm, as_stream(stream));
  });
}

int msx_csr_transpose(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
                      int64_t nnz, int64_t n_rows, int64_t n_cols, void *out_data, void *out_indices,
                      void *out_indptr, int64_t *out_perm, void *stream) {
  return guarded([&] {
    require(n_rows >= 0 && n_cols >= 0, MSX_ERR_INVALID, "csr_transpose shape dimensions must be non-negative.");
    require(nnz >= 0, MSX_ERR_INVALID, "csr_transpose nnz must be non-negative.");
    dispatch_value(value_dtype, [](auto) {});
    dispatch_index(index_dtype, [](auto) {});
    check_ptr(indices, nnz, "csr_transpose indices");
    check_ptr(indptr, n_rows + 1, "csr_transpose indptr");
    check_ptr(out_indices, nnz, "csr_transpose out_indices");
    check_ptr(out_indptr, n_cols + 1, "csr_transpose out_indptr");
    if (out_data) check_ptr(data, nnz, "csr_transpose data");
    csr_transpose_run(value_dtype, index_dtype, data, indices, indptr, nnz, n_rows, n_cols, out_data, out_indices,
                      out_indptr, out_perm, as_stream(stream));
  });
}

// A^T @ rhs (k = 0: rhs is a vector). Builds the transposed CSR in stream
// scratch, then runs the product kernels over it.
static void transposed_product(int value_dtype, int index_dtype, const void *data, const void *indices,
                               const void *indptr, int64_t nnz, const void *rhs, int64_t k, void *out,
                               int64_t n_rows, int64_t n_cols, cudaStream_t s) {
  if (n_cols == 0) return;
  size_t vb = 0, ib = index_dtype == MSX_I64 ? 8 : 4;
  dispatch_value(value_dtype, [&](auto v) { vb = sizeof(v); });
  Scratch t_data(vb * (size_t)nnz, s), t_idx(ib * (size_t)nnz, s), t_ptr(ib * (size_t)(n_cols + 1), s);
  csr_transpose_run(value_dtype, index_dtype, data, indices, indptr, nnz, n_rows, n_cols, t_data.ptr, t_idx.ptr,
                    t_ptr.ptr, nullptr, s);
  if (k == 0) {
    const int64_t n_tiles = spmv_num_tiles(n_cols, nnz);
    const size_t plan_bytes = spmv_plan_device_bytes(n_tiles);
    Scratch scratch(plan_bytes + sizeof(float) * 2 * n_tiles, s);
    char *base = scratch.as<char>();
    spmv_build_plan(index_dtype, t_ptr.ptr, n_cols, nnz, base, n_tiles, s);
    spmv_run(value_dtype, index_dtype, t_data.ptr, t_idx.ptr, t_ptr.ptr, rhs, out, n_cols, nnz, base, n_tiles, true,
             reinterpret_cast<float *>(base + plan_bytes), s);
  } else {
    spmm_run(value_dtype, index_dtype, t_data.ptr, t_idx.ptr, t_ptr.ptr, rhs, k, out, n_cols, n_rows, nnz, s);
  }
}

int msx_csr_matvec_transpose(int value_dtype, int index_dtype, const void *data, const void *indices,
                             const void *indptr, int64_t nnz, const void *x, void *out, int64_t n_rows,
                             int64_t n_cols, void *stream) {
  return guarded([&] {
    require(n_rows >= 0 && n_cols >= 0 && nnz >= 0, MSX_ERR_INVALID,
            "csr_matvec_transpose sizes must be non-negative.");
    check_ptr(data, nnz, "csr_matvec_transpose data");
    check_ptr(indices, nnz, "csr_matvec_transpose indices");
    check_ptr(indptr, n_rows + 1, "csr_matvec_transpose indptr");
    check_ptr(x, nnz > 0 ? n_rows : 0, "csr_matvec_transpose x");
    check_ptr(out, n_cols, "csr_matvec_transpose out");
    transposed_product(value_dtype, index_dtype, data, indices, indptr, nnz, x, 0, out, n_rows, n_cols,
                       as_stream(stream));
  });
}

int msx_csr_matmul_transpose(int value_dtype, int index_dtype, const void *data, const void *indices,
                             const void *indptr, int64_t nnz, const void *rhs, int64_t rhs_cols, void *out,
                             int64_t n_rows, int64_t n_cols, void *stream) {
  return guarded([&] {
    require(n_rows >= 0 && n_cols >= 0 && nnz >= 0 && rhs_cols >= 0, MSX_ERR_INVALID,
            "csr_matmul_transpose sizes must be non-negative.");
    check_ptr(data, nnz, "csr_matmul_transpose data");
    check_ptr(indices, nnz, "csr_matmul_transpose indices");
    check_ptr(indptr, n_rows + 1, "csr_matmul_transpose indptr");
    check_ptr(rhs, nnz > 0 ? n_rows * rhs_cols : 0, "csr_matmul_transpose rhs");
    check_ptr(out, n_cols * rhs_cols, "csr_matmul_transpose out");
    if (rhs_cols == 0) return;
    transposed_product(value_dtype, index_dtype, data, indices, indptr, nnz, rhs, rhs_cols, out, n_rows, n_cols,
                       as_stream(stream));
  });
}

int msx_csr_matmul_data_vjp(int value_dtype, int index_dtype, const void *indices, const void *indptr, int64_t nnz,
                            const void *rhs, const void *cotangent, int64_t rhs_cols, void *out, int64_t n_rows,
                            int64_t n_cols, void *stream) {
  return guarded([&] {
    require(n_rows >= 0 && n_cols >= 0 && nnz >= 0 && rhs_cols >= 0, MSX_ERR_INVALID,
            "csr_matmul_data_vjp sizes must be non-negative.");
    dispatch_value(value_dtype, [](auto) {});
    dispatch_index(index_dtype, [](auto) {});
    check_ptr(indices, nnz, "csr_matmul_data_vjp indices");
    check_ptr(indptr, n_rows + 1, "csr_matmul_data_vjp indptr");
    check_ptr(rhs, nnz > 0 ? n_cols * rhs_cols : 0, "csr_matmul_data_vjp rhs");
    check_ptr(cotangent, nnz > 0 ? n_rows * rhs_cols : 0, "csr_matmul_data_vjp cotangent");
    check_ptr(out, nnz, "csr_matmul_data_vjp out");
    csr_data_vjp_run(value_dtype, index_dtype, indices, indptr, nnz, n_rows, rhs, cotangent, rhs_cols, out,
                     as_stream(stream));
  });
}

int msx_csr_matvec_data_vjp(int value_dtype, int index_dtype, const void *indices, const void *indptr, int64_t nnz,
                            const void *x, const void *cotangent, void *out, int64_t n_rows, int64_t n_cols,
                            void *stream) {
  return msx_csr_matmul_data_vjp(value_dtype, index_dtype, indices, indptr, nnz, x, cotangent, 1, out, n_rows, n_cols,
                                 stream);
}

int msx_csr_batched_matvec(int value_dtype, int index_dtype, const void *data, const void *indices,
                           const void *indptr, int64_t nnz, const void *rhs, int64_t batch, void *out, int64_t n_rows,
                           int64_t n_cols, void *stream) {
  return guarded([&] {
    require(n_rows >= 0 && n_cols >= 0, MSX_ERR_INVALID, "csr_batched_matvec shape dimensions must be non-negative.");
    require(nnz >= 0 && batch >= 0, MSX_ERR_INVALID, "csr_batched_matvec sizes must be non-negative.");
    dispatch_value(value_dtype, [](auto) {});
    dispatch_index(index_dtype, [](auto) {});
    check_ptr(data, nnz, "csr_batched_matvec data");
    check_ptr(indices, nnz, "csr_batched_matvec indices");
    check_ptr(indptr, n_rows + 1, "csr_batched_matvec indptr");
    check_ptr(rhs, batch * n_cols, "csr_batched_matvec rhs");
    check_ptr(out, batch * n_rows, "csr_batched_matvec out");
    csr_batched_matvec_run(value_dtype, index_dtype, data, indices, indptr, nnz, n_rows, n_cols, batch, rhs, out,
                           as_stream(stream));
  });
}

int msx_csr_batched_matmul(int value_dtype, int index_dtype, const void *data, const void *indices,
                           const void *indptr, int64_t nnz, const void *rhs, int64_t batch, int64_t rhs_cols,
                           void *out, int64_t n_rows, int64_t n_cols, void *stream) {
  return guarded([&] {
    require(n_rows >= 0 && n_cols >= 0, MSX_ERR_INVALID, "csr_batched_matmul shape dimensions must be non-negative.");
    require(nnz >= 0 && batch >= 0 && rhs_cols >= 0, MSX_ERR_INVALID,
            "csr_batched_matmul sizes must be non-negative.");
    dispatch_value(value_dtype, [](auto) {});
    dispatch_index(index_dtype, [](auto) {});
    check_ptr(data, nnz, "csr_batched_matmul data");
    check_ptr(indices, nnz, "csr_batched_matmul indices");
    check_ptr(indptr, n_rows + 1, "csr_batched_matmul indptr");
    check_ptr(rhs, batch * n_cols * rhs_cols, "csr_batched_matmul rhs");
    check_ptr(out, batch * n_rows * rhs_cols, "csr_batched_matmul out");
    csr_batched_matmul_run(value_dtype, index_dtype, data, indices, indptr, nnz, n_rows, n_cols, batch, rhs_cols,
                           rhs, out, as_stream(stream));
  });
}

static void check_matmat_args(int value_dtype, int lit, const void *ld, const void *li, const void *lp,
                              int64_t lnnz, int rit, const void *rd, const void *ri, const void *rp, int64_t rnnz,
                              int64_t m, int64_t k, int64_t rk, int64_t n, int out_it) {
  require(m >= 0 && k >= 0 && rk >= 0 && n >= 0, MSX_ERR_INVALID, "csr_matmat shape dimensions must be non-negative.");
  require(k == rk, MSX_ERR_INVALID, "CSR sparse-sparse matmul dimension mismatch.");
  require(lnnz >= 0 && rnnz >= 0, MSX_ERR_INVALID, "csr_matmat nnz must be non-negative.");
  require(n <= (int64_t)INT32_MAX, MSX_ERR_OVERFLOW, "csr_matmat n_cols exceeds supported limits.");
  dispatch_value(value_dtype, [](auto) {});
  dispatch_index(lit, [](auto) {});
  dispatch_index(rit, [](auto) {});
  dispatch_index(out_it, [](auto) {});
  require(out_it == (lit == rit ? lit : (int)MSX_I64), MSX_ERR_TYPE,
          "csr_matmat output index dtype must be the inputs' when they agree, else int64.");
  check_ptr(ld, lnnz, "csr_matmat lhs_data");
  check_ptr(li, lnnz, "csr_matmat lhs_indices");
  check_ptr(lp, m + 1, "csr_matmat lhs_indptr");
  check_ptr(rd, rnnz, "csr_matmat rhs_data");
  check_ptr(ri, rnnz, "csr_matmat rhs_indices");
  check_ptr(rp, rk + 1, "csr_matmat rhs_indptr");
}

int msx_csr_matmat_symbolic(int value_dtype, int lhs_index_dtype, const void *lhs_data, const void *lhs_indices,
                            const void *lhs_indptr, int64_t lhs_nnz, int rhs_index_dtype, const void *rhs_data,
                            const void *rhs_indices, const void *rhs_indptr, int64_t rhs_nnz, int64_t lhs_n_rows,
                            int64_t lhs_n_cols, int64_t rhs_n_rows, int64_t rhs_n_cols, int out_index_dtype,
                            void *out_indptr, int64_t *out_nnz, int prune_zeros, void *stream) {
  return guarded([&] {
    check_matmat_args(value_dtype, lhs_index_dtype, lhs_data, lhs_indices, lhs_indptr, lhs_nnz, rhs_index_dtype,
                      rhs_data, rhs_indices, rhs_indptr, rhs_nnz, lhs_n_rows, lhs_n_cols, rhs_n_rows, rhs_n_cols,
                      out_index_dtype);
    require(out_nnz != nullptr, MSX_ERR_INVALID, "csr_matmat out_nnz must not be null.");
    check_ptr(out_indptr, lhs_n_rows + 1, "csr_matmat out_indptr");
    spgemm_run(false, value_dtype, lhs_index_dtype, lhs_data, lhs_indices, lhs_indptr, rhs_index_dtype, rhs_data,
               rhs_indices, rhs_indptr, lhs_n_rows, rhs_n_rows, rhs_n_cols, out_index_dtype, out_indptr, nullptr,
               nullptr, out_nnz, prune_zeros != 0, as_stream(stream));
  });
}

int msx_csr_matmat_numeric(int value_dtype, int lhs_index_dtype, const void *lhs_data, const void *lhs_indices,
                           const void *lhs_indptr, int64_t lhs_nnz, int rhs_index_dtype, const void *rhs_data,
                           const void *rhs_indices, const void *rhs_indptr, int64_t rhs_nnz, int64_t lhs_n_rows,
                           int64_t lhs_n_cols, int64_t rhs_n_rows, int64_t rhs_n_cols, int out_index_dtype,
                           const void *out_indptr, int64_t out_nnz, void *out_data, void *out_indices,
                           int prune_zeros, void *stream) {
  return guarded([&] {
    check_matmat_args(value_dtype, lhs_index_dtype, lhs_data, lhs_indices, lhs_indptr, lhs_nnz, rhs_index_dtype,
                      rhs_data, rhs_indices, rhs_indptr, rhs_nnz, lhs_n_rows, lhs_n_cols, rhs_n_rows, rhs_n_cols,
                      out_index_dtype);
    require(out_nnz >= 0, MSX_ERR_INVALID, "csr_matmat out_nnz must be non-negative.");
    check_ptr(out_indptr, lhs_n_rows + 1, "csr_matmat out_indptr");
    check_ptr(out_data, out_nnz, "csr_matmat out_data");
    check_ptr(out_indices, out_nnz, "csr_matmat out_indices");
    int64_t capacity = out_nnz;
    spgemm_run(true, value_dtype, lhs_index_dtype, lhs_data, lhs_indices, lhs_indptr, rhs_index_dtype, rhs_data,
               rhs_indices, rhs_indptr, lhs_n_rows, rhs_n_rows, rhs_n_cols, out_index_dtype,
               const_cast<void *>(out_indptr), out_indices, out_data, &capacity, prune_zeros != 0,
               as_stream(stream));
  });
}

static void check_solver_args(const char *op, int index_dtype, const float *data, const void *indices,
                              const void *indptr, int64_t nnz, const float *b, const float *x0, float *x_out,
                              int64_t n_rows, int64_t n_cols, int32_t maxiter, int32_t *info, float *residual,
                              int32_t *iterations) {
  const std::string o(op);
  require(n_rows > 0 && n_cols > 0 && n_rows == n_cols, MSX_ERR_INVALID, o + " requires a non-empty square matrix.");
  require(maxiter >= 0, MSX_ERR_INVALID, o + " maxiter must be non-negative.");
  require(nnz >= 0, MSX_ERR_INVALID, o + " data and indices must have equal length.");
  dispatch_index(index_dtype, [](auto) {});
  check_ptr(data, nnz, (o + " data").c_str());
  check_ptr(indices, nnz, (o + " indices").c_str());
  check_ptr(indptr, n_rows + 1, (o + " indptr").c_str());
  check_ptr(b, n_rows, (o + " b").c_str());
  check_ptr(x0, n_cols, (o + " x0").c_str());
  check_ptr(x_out, n_rows, (o + " x").c_str());
  require(info && residual && iterations, MSX_ERR_INVALID, o + " result pointers must not be null.");
}

int msx_csr_cg(int index_dtype, const float *data, const void *indices, const void *indptr, int64_t nnz,
               const float *b, const float *x0, float *x_out, int64_t n_rows, int64_t n_cols, float rtol, float atol,
               int32_t maxiter, int32_t *info, float *residual, int32_t *iterations, void *stream) {
  return guarded([&] {
    check_solver_args("csr_cg", index_dtype, data, indices, indptr, nnz, b, x0, x_out, n_rows, n_cols, maxiter,
                      info, residual, iterations);
    CgProblem prob{index_dtype, data, indices, indptr, nnz, n_rows, n_cols, b, x0, nullptr, x_out, rtol, atol,
                   maxiter};
    CgResult r = cg_solve(prob, as_stream(stream));
    *info = r.info;
    *residual = r.residual;
    *iterations = r.iterations;
  });
}

int msx_csr_pcg_jacobi(int index_dtype, const float *data, const void *indices, const void *indptr, int64_t nnz,
                       const float *b, const float *x0, const float *inv_diag, float *x_out, int64_t n_rows,
                       int64_t n_cols, float rtol, float atol, int32_t maxiter, int32_t *info, float *residual,
                       int32_t *iterations, void *stream) {
  return guarded([&] {
    check_solver_args("csr_pcg_jacobi", index_dtype, data, indices, indptr, nnz, b, x0, x_out, n_rows, n_cols,
                      maxiter, info, residual, iterations);
    check_ptr(inv_diag, n_rows, "csr_pcg_jacobi inv_diag");
    CgProblem prob{index_dtype, data, indices, indptr, nnz, n_rows, n_cols, b, x0, inv_diag, x_out, rtol, atol,
                   maxiter};
    CgResult r = cg_solve(prob, as_stream(stream));
    *info = r.info;
    *residual = r.residual;
    *iterations = r.iterations;
  });
}

static void check_chebyshev(const char *op, int degree, float lambda_min, float lambda_max) {
  // validate_chebyshev_interval, src/preconditioners/pcg/chebyshev.cpp:66-78
  if (degree <= 0) fail(MSX_ERR_INVALID, std::string(op) + " degree must be positive.");
  if (!std::isfinite(lambda_min) || !std::isfinite(lambda_max) || lambda_min <= 0.0f || lambda_max <= lambda_min)
    fail(MSX_ERR_INVALID, std::string(op) + " requires finite bounds satisfying 0 < lambda_min < lambda_max.");
}

int msx_csr_pcg_chebyshev(int index_dtype, const float *data, const void *indices, const void *indptr, int64_t nnz,
                          const float *b, const float *x0, const float *m_data, const void *m_indices,
                          const void *m_indptr, int64_t m_nnz, float *x_out, int64_t n_rows, int64_t n_cols,
                          int32_t degree, float lambda_min, float lambda_max, float rtol, float atol,
                          int32_t maxiter, int32_t *info, float *residual, int32_t *iterations, void *stream) {
  return guarded([&] {
    check_solver_args("csr_pcg_chebyshev", index_dtype, data, indices, indptr, nnz, b, x0, x_out, n_rows, n_cols,
                      maxiter, info, residual, iterations);
    check_chebyshev("csr_pcg_chebyshev", degree, lambda_min, lambda_max);
    require(m_nnz >= 0, MSX_ERR_INVALID, "csr_pcg_chebyshev preconditioner nnz must be non-negative.");
    check_ptr(m_data, m_nnz, "csr_pcg_chebyshev m_data");
    check_ptr(m_indices, m_nnz, "csr_pcg_chebyshev m_indices");
    check_ptr(m_indptr, n_rows + 1, "csr_pcg_chebyshev m_indptr");
    CgProblem prob{index_dtype, data, indices, indptr, nnz, n_rows, n_cols, b, x0, nullptr, x_out, rtol, atol,
                   maxiter};
    prob.m_data = m_data;
    prob.m_indices = m_indices;
    prob.m_indptr = m_indptr;
    prob.m_nnz = m_nnz;
    prob.degree = degree;
    prob.lambda_min = lambda_min;
    prob.lambda_max = lambda_max;
    CgResult r = cg_solve(prob, as_stream(stream));
    *info = r.info;
    *residual = r.residual;
    *iterations = r.iterations;
  });
}

int msx_csr_chebyshev_apply(int index_dtype, const float *m_data, const void *m_indices, const void *m_indptr,
                            int64_t m_nnz, int64_t n, const float *rhs, int64_t rhs_cols, float *out,
                            int32_t degree, float lambda_min, float lambda_max, void *stream) {
  return guarded([&] {
    require(n > 0 && m_nnz >= 0, MSX_ERR_INVALID,
            "csr_chebyshev_preconditioner_apply requires a non-empty square matrix.");
    require(rhs_cols > 0, MSX_ERR_INVALID, "csr_chebyshev_preconditioner_apply rhs must have at least one column.");
    dispatch_index(index_dtype, [](auto) {});
    check_chebyshev("csr_chebyshev_preconditioner_apply", degree, lambda_min, lambda_max);
    check_ptr(m_data, m_nnz, "csr_chebyshev_preconditioner_apply data");
    check_ptr(m_indices, m_nnz, "csr_chebyshev_preconditioner_apply indices");
    check_ptr(m_indptr, n + 1, "csr_chebyshev_preconditioner_apply indptr");
    check_ptr(rhs, n * rhs_cols, "csr_chebyshev_preconditioner_apply rhs");
    check_ptr(out, n * rhs_cols, "csr_chebyshev_preconditioner_apply out");
    chebyshev_apply_run(index_dtype, m_data, m_indices, m_indptr, m_nnz, n, rhs, rhs_cols, out, degree, lambda_min,
                        lambda_max, as_stream(stream));
  });
}

int msx_diagonal_preconditioner_apply(const float *inv_diag, const float *rhs, int64_t n, int64_t rhs_cols,
                                      float *out, void *stream) {
  return guarded([&] {
    require(n >= 0, MSX_ERR_INVALID, "diagonal_preconditioner_apply sizes must be non-negative.");
    require(rhs_cols > 0, MSX_ERR_INVALID, "diagonal_preconditioner_apply rhs must have at least one column.");
    check_ptr(inv_diag, n, "diagonal_preconditioner_apply inv_diag");
    check_ptr(rhs, n * rhs_cols, "diagonal_preconditioner_apply rhs");
    check_ptr(out, n * rhs_cols, "diagonal_preconditioner_apply out");
    diagonal_apply_run(inv_diag, rhs, n, rhs_cols, out, as_stream(stream));
  });
}

int msx_csr_gershgorin_bounds(int index_dtype, const float *data, const void *indices, const void *indptr,
                              int64_t nnz, int64_t n_rows, int64_t n_cols, float *out4, void *stream) {
  return guarded([&] {
    require(n_rows > 0 && n_rows == n_cols, MSX_ERR_INVALID,
            "csr_chebyshev_spectral_bounds requires a non-empty square matrix.");
    dispatch_index(index_dtype, [](auto) {});
    check_ptr(data, nnz, "csr_chebyshev_spectral_bounds data");
    check_ptr(indices, nnz, "csr_chebyshev_spectral_bounds indices");
    check_ptr(indptr, n_rows + 1, "csr_chebyshev_spectral_bounds indptr");
    require(out4 != nullptr, MSX_ERR_INVALID, "csr_chebyshev_spectral_bounds out must not be null.");
    gershgorin_run(index_dtype, data, indices, indptr, n_rows, out4, as_stream(stream));
  });
}

int msx_csr_diagonal(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
                     int64_t nnz, int64_t n_rows, int64_t n_cols, void *out, void *stream) {
  return guarded([&] {
    require(n_rows >= 0 && n_cols >= 0 && nnz >= 0, MSX_ERR_INVALID, "csr_diagonal sizes must be non-negative.");
    dispatch_value(value_dtype, [](auto) {});
    dispatch_index(index_dtype, [](auto) {});
    const int64_t n_diag = n_rows < n_cols ? n_rows : n_cols;
    check_ptr(data, nnz, "csr_diagonal data");
    check_ptr(indices, nnz, "csr_diagonal indices");
    check_ptr(indptr, n_rows + 1, "csr_diagonal indptr");
    check_ptr(out, n_diag, "csr_diagonal out");
    csr_diagonal_run(value_dtype, index_dtype, data, indices, indptr, n_diag, out, as_stream(stream));
  });
}

// ---- multi-GPU (NCCL) ---------------------------------------------------------
int msx_dist_unique_id(void *out, int64_t size) {
  return guarded([&] {
#if defined(MSX_HAVE_NCCL)
    require(out != nullptr && size >= (int64_t)sizeof(ncclUniqueId), MSX_ERR_INVALID,
            "msx_dist_unique_id needs a buffer of at least 128 bytes.");
    ncclUniqueId id;
    const ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) fail(MSX_ERR_RUNTIME, std::string("ncclGetUniqueId: ") + ncclGetErrorString(r));
    std::memcpy(out, &id, sizeof(id));
#else
    (void)out;
    (void)size;
    fail(MSX_ERR_RUNTIME, "this build has no NCCL.");
#endif
  });
}

int msx_dist_comm_create(const void *unique_id, int nranks, int rank, void **out) {
  return guarded([&] {
#if defined(MSX_HAVE_NCCL)
    require(unique_id && out, MSX_ERR_INVALID, "msx_dist_comm_create: null argument.");
    require(nranks > 0 && rank >= 0 && rank < nranks, MSX_ERR_INVALID, "msx_dist_comm_create: bad rank.");
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    ncclComm_t comm;
    const ncclResult_t r = ncclCommInitRank(&comm, nranks, id, rank);
    if (r != ncclSuccess) fail(MSX_ERR_RUNTIME, std::string("ncclCommInitRank: ") + ncclGetErrorString(r));
    *out = comm;
#else
    (void)unique_id;
    (void)nranks;
    (void)rank;
    (void)out;
    fail(MSX_ERR_RUNTIME, "this build has no NCCL.");
#endif
  });
}

int msx_dist_comm_destroy(void *comm) {
  return guarded([&] {
#if defined(MSX_HAVE_NCCL)
    if (comm) ncclCommDestroy(static_cast<ncclComm_t>(comm));
#else
    (void)comm;
#endif
  });
}

int msx_dist_pcg(void *comm, int index_dtype, const float *data, const void *indices, const void *indptr,
                 int64_t nnz, int64_t n_owned, int64_t n_halo, const float *b, const float *x0,
                 const float *inv_diag, float *x_out, float rtol, float atol, int32_t maxiter, int n_peers,
                 const int *peers, const int64_t *send_counts, const int64_t *recv_counts, const int *send_idx,
                 int32_t *info, float *residual, int32_t *iterations, void *stream) {
  return guarded([&] {
    require(comm != nullptr, MSX_ERR_INVALID, "msx_dist_pcg: comm must not be null.");
    require(n_owned > 0 && n_halo >= 0 && n_peers >= 0, MSX_ERR_INVALID, "msx_dist_pcg: bad sizes.");
    require(maxiter >= 0, MSX_ERR_INVALID, "csr_cg maxiter must be non-negative.");
    require(n_peers == 0 || (peers && send_counts && recv_counts), MSX_ERR_INVALID,
            "msx_dist_pcg: peer lists must not be null.");
    dispatch_index(index_dtype, [](auto) {});
    check_ptr(data, nnz, "csr_cg data");
    check_ptr(indices, nnz, "csr_cg indices");
    check_ptr(indptr, n_owned + 1, "csr_cg indptr");
    check_ptr(b, n_owned, "csr_cg b");
    check_ptr(x0, n_owned, "csr_cg x0");
    check_ptr(x_out, n_owned, "csr_cg x");
    require(info && residual && iterations, MSX_ERR_INVALID, "csr_cg result pointers must not be null.");
    CgDist d{comm, n_peers, peers, send_counts, recv_counts, send_idx, n_halo};
    CgProblem prob{index_dtype, data, indices, indptr, nnz, n_owned, n_owned + n_halo, b, x0, inv_diag, x_out,
                   rtol, atol, maxiter, &d};
    CgResult r = cg_solve(prob, as_stream(stream));
    *info = r.info;
    *residual = r.residual;
    *iterations = r.iterations;
  });
}

// ---- persistent CG contexts ------------------------------------------------------
int msx_cg_context_create(int index_dtype, const float *data, const void *indices, const void *indptr, int64_t nnz,
                          int64_t n_owned, int64_t n_halo, int preconditioned, int comm_mode, int rank, int world,
                          void *nccl_comm, int n_peers, const int *peers, const int64_t *send_counts,
                          const int64_t *recv_counts, const int *send_idx, const int64_t *peer_dst_offset,
                          void *stream, msx_cg_context **out) {
  return guarded([&] {
    require(out != nullptr, MSX_ERR_INVALID, "msx_cg_context_create: out must not be null.");
    *out = nullptr;
    require(n_owned > 0 && n_halo >= 0 && nnz >= 0, MSX_ERR_INVALID, "csr_cg requires a non-empty square matrix.");
    require(world >= 1 && world <= kMaxRanks && rank >= 0 && rank < world, MSX_ERR_INVALID, "bad rank / world.");
    require(comm_mode >= kCommNone && comm_mode <= kCommP2p, MSX_ERR_INVALID, "bad comm mode.");
    require(world == 1 || comm_mode != kCommNone, MSX_ERR_INVALID, "multi-rank contexts need a comm mode.");
    require(comm_mode != kCommNccl || nccl_comm, MSX_ERR_INVALID, "NCCL mode needs a communicator.");
    require(n_peers >= 0 && n_peers < kMaxRanks, MSX_ERR_INVALID, "bad peer count.");
    require(n_peers == 0 || (peers && send_counts && recv_counts), MSX_ERR_INVALID, "peer lists must not be null.");
    require(comm_mode != kCommP2p || n_peers == 0 || peer_dst_offset, MSX_ERR_INVALID,
            "P2P mode needs the landing offsets.");
    int64_t n_send = 0;
    for (int k = 0; k < n_peers; ++k) {
      require(send_counts[k] >= 0 && recv_counts[k] >= 0, MSX_ERR_INVALID, "peer counts must be non-negative.");
      n_send += send_counts[k];
    }
    require(n_send == 0 || send_idx, MSX_ERR_INVALID, "send_idx must not be null when entries are sent.");
    dispatch_index(index_dtype, [](auto) {});
    check_ptr(data, nnz, "csr_cg data");
    check_ptr(indices, nnz, "csr_cg indices");
    check_ptr(indptr, n_owned + 1, "csr_cg indptr");
    std::unique_ptr<msx_cg_context> ctx(new msx_cg_context());
    ctx->world = world;
    ctx->peers.assign(peers, peers + n_peers);
    ctx->send_counts.assign(send_counts, send_counts + n_peers);
    ctx->recv_counts.assign(recv_counts, recv_counts + n_peers);
    if (peer_dst_offset) ctx->dst_offset.assign(peer_dst_offset, peer_dst_offset + n_peers);
    CgEngineConfig cfg{};
    cfg.index_dtype = index_dtype;
    cfg.data = data;
    cfg.indices = indices;
    cfg.indptr = indptr;
    cfg.nnz = nnz;
    cfg.n = n_owned;
    cfg.n_halo = n_halo;
    cfg.preconditioned = preconditioned != 0;
    cfg.comm = comm_mode;
    cfg.rank = rank;
    cfg.world = world;
    cfg.nccl_comm = nccl_comm;
    cfg.n_peers = n_peers;
    cfg.peers = ctx->peers.data();
    cfg.send_counts = ctx->send_counts.data();
    cfg.recv_counts = ctx->recv_counts.data();
    cfg.send_idx = send_idx;
    cfg.peer_dst_offset = ctx->dst_offset.empty() ? nullptr : ctx->dst_offset.data();
    ctx->engine = cg_engine_create(cfg, as_stream(stream));
    *out = ctx.release();
  });
}

static_assert(MSX_CG_IPC_BYTES == msx::kCgIpcBytes, "IPC descriptor size");

int msx_cg_context_ipc_handles(msx_cg_context *ctx, void *out, int64_t size) {
  return guarded([&] {
    require(ctx && out && size >= MSX_CG_IPC_BYTES, MSX_ERR_INVALID,
            "msx_cg_context_ipc_handles needs a buffer of MSX_CG_IPC_BYTES.");
    cg_engine_ipc_handles(ctx->engine, out);
  });
}

int msx_cg_context_connect(msx_cg_context *ctx, const void *all_handles, int64_t size) {
  return guarded([&] {
    require(ctx && all_handles, MSX_ERR_INVALID, "msx_cg_context_connect: null argument.");
    require(size >= MSX_CG_IPC_BYTES * (int64_t)ctx->world, MSX_ERR_INVALID,
            "msx_cg_context_connect: need world x MSX_CG_IPC_BYTES bytes.");
    cg_engine_connect(ctx->engine, all_handles);
  });
}

int msx_cg_context_solve(msx_cg_context *ctx, const float *b, const float *x0, const float *inv_diag, float *x_out,
                         float rtol, float atol, int32_t maxiter, int32_t *info, float *residual, int32_t *iterations,
                         void *stream) {
  return guarded([&] {
    require(ctx != nullptr, MSX_ERR_INVALID, "context must not be null.");
    require(maxiter >= 0, MSX_ERR_INVALID, "csr_cg maxiter must be non-negative.");
    require(b && x0 && x_out && info && residual && iterations, MSX_ERR_INVALID, "csr_cg: null argument.");
    CgResult r = cg_engine_solve(ctx->engine, b, x0, inv_diag, x_out, rtol, atol, maxiter, as_stream(stream));
    *info = r.info;
    *residual = r.residual;
    *iterations = r.iterations;
  });
}

int msx_cg_context_destroy(msx_cg_context *ctx) {
  return guarded([&] { delete ctx; });
}

}  // extern "C"
