// C-ABI entry points (include/msx_sparse.h). Argument checks follow the
// reference front-ends (e.g. src/sparse/csr_matvec/csr_matvec.cpp:326-356) and
// map C++ exception kinds onto msx_status codes.
#include <mutex>
#include <string>

#include "msx_sparse.h"
#include "ops.cuh"
#include "spmv.cuh"

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
  void *dev = nullptr;
  int device = 0;
  int64_t n_rows = 0;
  int64_t nnz = 0;
  int64_t n_tiles = 0;
  int64_t n_split = 0;
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

int msx_spmv_plan_create(int index_dtype, const void *indptr, int64_t n_rows, int64_t nnz, void *stream,
                         msx_spmv_plan **out) {
  return guarded([&] {
    require(out != nullptr, MSX_ERR_INVALID, "msx_spmv_plan_create: out must not be null.");
    *out = nullptr;
    require(n_rows >= 0 && nnz >= 0, MSX_ERR_INVALID, "csr_matvec shape dimensions must be non-negative.");
    check_ptr(indptr, n_rows + 1, "csr_matvec indptr");
    dispatch_index(index_dtype, [](auto) {});
    auto *plan = new msx_spmv_plan();
    plan->n_rows = n_rows;
    plan->nnz = nnz;
    plan->n_tiles = spmv_num_tiles(n_rows, nnz);
    MSX_CUDA(cudaGetDevice(&plan->device));
    cudaError_t e = cudaMalloc(&plan->dev, spmv_plan_device_bytes(plan->n_tiles));
    if (e != cudaSuccess) {
      delete plan;
      fail(MSX_ERR_CUDA, std::string("cudaMalloc for the SpMV plan failed: ") + cudaGetErrorString(e));
    }
    try {
      cudaStream_t s = as_stream(stream);
      spmv_build_plan(index_dtype, indptr, n_rows, nnz, plan->dev, plan->n_tiles, s);
      unsigned long long split = 0;
      int64_t *tr, *tn;
      unsigned long long *ns;
      spmv_plan_layout(plan->dev, plan->n_tiles, &tr, &tn, &ns);
      MSX_CUDA(cudaMemcpyAsync(&split, ns, sizeof(split), cudaMemcpyDeviceToHost, s));
      MSX_CUDA(cudaStreamSynchronize(s));
      plan->n_split = (int64_t)split;
    } catch (...) {
      cudaFree(plan->dev);
      delete plan;
      throw;
    }
    *out = plan;
  });
}

int msx_spmv_plan_destroy(msx_spmv_plan *plan) {
  return guarded([&] {
    if (!plan) return;
    if (plan->dev) {
      int cur = 0;
      cudaGetDevice(&cur);
      if (cur != plan->device) cudaSetDevice(plan->device);
      cudaFree(plan->dev);
      if (cur != plan->device) cudaSetDevice(cur);
    }
    delete plan;
  });
}

int msx_spmv_plan_info(const msx_spmv_plan *plan, int64_t *n_tiles, int64_t *n_split_boundaries) {
  return guarded([&] {
    require(plan != nullptr, MSX_ERR_INVALID, "plan must not be null.");
    if (n_tiles) *n_tiles = plan->n_tiles;
    if (n_split_boundaries) *n_split_boundaries = plan->n_split;
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
      require(plan->n_rows == n_rows && plan->nnz == nnz, MSX_ERR_INVALID,
              "csr_matvec plan was built for a different matrix shape.");
      if (plan->n_split > 0) {
        Scratch carry(sizeof(float) * 2 * plan->n_tiles, s);
        spmv_run(value_dtype, index_dtype, data, indices, indptr, x, y, n_rows, plan->dev, plan->n_tiles, true,
                 carry.as<float>(), s);
      } else {
        spmv_run(value_dtype, index_dtype, data, indices, indptr, x, y, n_rows, plan->dev, plan->n_tiles, false,
                 nullptr, s);
      }
      return;
    }
    const int64_t n_tiles = spmv_num_tiles(n_rows, nnz);
    const size_t plan_bytes = spmv_plan_device_bytes(n_tiles);
    Scratch scratch(plan_bytes + sizeof(float) * 2 * n_tiles, s);
    char *base = scratch.as<char>();
    spmv_build_plan(index_dtype, indptr, n_rows, nnz, base, n_tiles, s);
    spmv_run(value_dtype, index_dtype, data, indices, indptr, x, y, n_rows, base, n_tiles, true,
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
    spmm_run(value_dtype, index_dtype, data, indices, indptr, rhs, rhs_cols, out, n_rows, n_cols,
             as_stream(stream));
  });
}

}  // extern "C"
