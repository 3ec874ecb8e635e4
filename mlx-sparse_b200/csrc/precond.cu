// Preconditioner applications and spectral bounds outside the solve loop.
//
// Reference behaviour:
//  - diagonal_preconditioner_apply (src/preconditioners/diagonal/
//    diagonal.cpp:60-88): out[row, c] = inv_diag[row] * rhs[row, c];
//  - csr_chebyshev_preconditioner_apply (src/preconditioners/chebyshev/
//    chebyshev.cpp:262-300): the first-kind Chebyshev semi-iteration of
//    `degree` terms with a zero start, column by column;
//  - the Gershgorin and diagonal bounds of csr_chebyshev_spectral_bounds
//    (chebyshev.cpp:120-161): per row, diag - sum|offdiag| and
//    diag + sum|offdiag| in double, min / max over rows.
//
// All three are HBM-bound streams. The Chebyshev apply uses the SpMM kernel
// for M @ out (k columns; k = 1 is a vector) and one fused update kernel per
// step, so every element follows the reference's float arithmetic.
#include <algorithm>
#include <cmath>
#include <limits>
#include <vector>

#include "cg.cuh"
#include "ops.cuh"

namespace msx {

namespace {

constexpr int kThreads = 256;

int grid_for(int64_t n) {
  const int64_t cap = (int64_t)num_sms() * 8;
  return (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(n, kThreads), cap));
}

__global__ void scale_rows_kernel(const float *__restrict__ inv, const float *__restrict__ rhs, int64_t n, int64_t k,
                                  float *__restrict__ out) {
  const int64_t total = n * k;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = __fmul_rn(inv[k == 1 ? i : i / k], rhs[i]);
}

__global__ void cheb_first(const float *__restrict__ rhs, float *__restrict__ out, float *__restrict__ prev,
                           int64_t total, float scale) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    out[i] = __fmul_rn(scale, rhs[i]);
    if (prev) prev[i] = 0.0f;
  }
}

__global__ void cheb_step(const float *__restrict__ rhs, const float *__restrict__ ax, const float *__restrict__ prev,
                          const float *__restrict__ out, float *__restrict__ next, int64_t total, float one_minus_omega,
                          float omega, float omega_scale) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const float rv = __fsub_rn(rhs[i], ax[i]);
    next[i] = __fadd_rn(__fadd_rn(__fmul_rn(one_minus_omega, prev[i]), __fmul_rn(omega, out[i])),
                        __fmul_rn(omega_scale, rv));
  }
}

__global__ void copy_kernel(const float *__restrict__ src, float *__restrict__ dst, int64_t total) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

// Per CTA: {min(diag - off), max(diag + off), min diag, max diag} and a
// non-finite count, from one thread per row.
template <typename I>
__global__ void __launch_bounds__(kThreads)
gershgorin_kernel(const float *__restrict__ data, const I *__restrict__ indices, const I *__restrict__ indptr,
                  int64_t n_rows, double *__restrict__ part) {
  __shared__ double sm[5][kThreads];
  const double inf = __longlong_as_double(0x7ff0000000000000ll);
  double lo = inf, hi = -inf, dmin = inf, dmax = -inf, bad = 0.0;
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < n_rows; r += (int64_t)gridDim.x * blockDim.x) {
    double diag = 0.0, off = 0.0;
    for (int64_t p = (int64_t)indptr[r]; p < (int64_t)indptr[r + 1]; ++p) {
      const float v = data[p];
      if (!isfinite(v)) bad += 1.0;
      if ((int64_t)indices[p] == r) diag += (double)v;
      else off += fabs((double)v);
    }
    lo = fmin(lo, diag - off);
    hi = fmax(hi, diag + off);
    dmin = fmin(dmin, diag);
    dmax = fmax(dmax, diag);
  }
  sm[0][threadIdx.x] = lo;
  sm[1][threadIdx.x] = hi;
  sm[2][threadIdx.x] = dmin;
  sm[3][threadIdx.x] = dmax;
  sm[4][threadIdx.x] = bad;
  __syncthreads();
  for (int w = kThreads / 2; w > 0; w >>= 1) {
    if (threadIdx.x < w) {
      sm[0][threadIdx.x] = fmin(sm[0][threadIdx.x], sm[0][threadIdx.x + w]);
      sm[1][threadIdx.x] = fmax(sm[1][threadIdx.x], sm[1][threadIdx.x + w]);
      sm[2][threadIdx.x] = fmin(sm[2][threadIdx.x], sm[2][threadIdx.x + w]);
      sm[3][threadIdx.x] = fmax(sm[3][threadIdx.x], sm[3][threadIdx.x + w]);
      sm[4][threadIdx.x] += sm[4][threadIdx.x + w];
    }
    __syncthreads();
  }
  if (threadIdx.x < 5) part[blockIdx.x * 5 + threadIdx.x] = sm[threadIdx.x][0];
}

}  // namespace

void diagonal_apply_run(const float *inv_diag, const float *rhs, int64_t n, int64_t k, float *out,
                        cudaStream_t stream) {
  if (n * k == 0) return;
  scale_rows_kernel<<<grid_for(n * k), kThreads, 0, stream>>>(inv_diag, rhs, n, k, out);
  MSX_CHECK_LAUNCH();
}

void chebyshev_apply_run(int index_dtype, const float *m_data, const void *m_indices, const void *m_indptr,
                         int64_t m_nnz, int64_t n, const float *rhs, int64_t k, float *out, int degree,
                         float lambda_min, float lambda_max, cudaStream_t s) {
  const int64_t total = n * k;
  if (total == 0) return;
  const float scale = 2.0f / (lambda_max + lambda_min);
  const float alpha = 1.0f - scale * lambda_min;
  const float mu = 1.0f / alpha;
  const float omega_prod = 2.0f / alpha;
  float c_prev = 1.0f, c_cur = mu;
  const int g = grid_for(total);
  Scratch work(sizeof(float) * (size_t)total * (degree > 1 ? 3 : 0), s);
  float *cur = out, *prev = nullptr, *next = nullptr, *ax = nullptr;
  if (degree > 1) {
    prev = work.as<float>();
    next = prev + total;
    ax = next + total;
  }
  cheb_first<<<g, kThreads, 0, s>>>(rhs, cur, prev, total, scale);
  MSX_CHECK_LAUNCH();
  for (int it = 1; it < degree; ++it) {
    spmm_run(MSX_F32, index_dtype, m_data, m_indices, m_indptr, cur, k, ax, n, n, m_nnz, s);
    const float c_next = 2.0f * mu * c_cur - c_prev;
    const float omega = omega_prod * c_cur / c_next;
    cheb_step<<<g, kThreads, 0, s>>>(rhs, ax, prev, cur, next, total, 1.0f - omega, omega, omega * scale);
    MSX_CHECK_LAUNCH();
    float *t = prev;
    prev = cur;
    cur = next;
    next = t;
    c_prev = c_cur;
    c_cur = c_next;
  }
  if (cur != out) {
    copy_kernel<<<g, kThreads, 0, s>>>(cur, out, total);
    MSX_CHECK_LAUNCH();
  }
}

void gershgorin_run(int index_dtype, const float *data, const void *indices, const void *indptr, int64_t n_rows,
                    float *out4, cudaStream_t s) {
  const int g = grid_for(n_rows);
  Scratch part(sizeof(double) * 5 * (size_t)g, s);
  dispatch_index(index_dtype, [&](auto ityp) {
    using I = decltype(ityp);
    gershgorin_kernel<I><<<g, kThreads, 0, s>>>(data, static_cast<const I *>(indices),
                                                 static_cast<const I *>(indptr), n_rows, part.as<double>());
  });
  MSX_CHECK_LAUNCH();
  std::vector<double> h(5 * (size_t)g);
  MSX_CUDA(cudaMemcpyAsync(h.data(), part.ptr, sizeof(double) * h.size(), cudaMemcpyDeviceToHost, s));
  MSX_CUDA(cudaStreamSynchronize(s));
  double lo = std::numeric_limits<double>::infinity(), hi = -lo, dmin = lo, dmax = -lo, bad = 0.0;
  for (int b = 0; b < g; ++b) {
    lo = std::min(lo, h[5 * b]);
    hi = std::max(hi, h[5 * b + 1]);
    dmin = std::min(dmin, h[5 * b + 2]);
    dmax = std::max(dmax, h[5 * b + 3]);
    bad += h[5 * b + 4];
  }
  if (bad != 0.0) fail(MSX_ERR_INVALID, "csr_chebyshev_spectral_bounds input contains a non-finite value.");
  out4[0] = (float)lo;
  out4[1] = (float)hi;
  out4[2] = (float)dmin;
  out4[3] = (float)dmax;
}

}  // namespace msx
