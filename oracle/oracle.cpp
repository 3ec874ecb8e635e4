// TEST INFRASTRUCTURE ONLY - the CPU oracle for the sparse-product hot path.
//
// A plain C++ restatement of mlx-sparse's CPU loops, used by tests/ to check
// the CUDA library and by bench.py as the timed CPU baseline. Nothing in the
// product path links or calls this file. Citations are relative to the
// mlx-sparse source tree:
//   SpMV      src/sparse/csr_matvec/csr_matvec.cpp:79-168
//   SpMM      src/sparse/csr_matmul/csr_matmul.cpp:83-222
//   SpGEMM    src/sparse/csr_matmat/csr_matmat.cpp:418-650 (serial host path;
//             the parallel path :652-817 produces identical output)
//   CG        src/linalg/cg/cg.cpp:75-256 with src/linalg/common/common.h:35-59
//   PCG       src/preconditioners/pcg/pcg.cpp:70-230
//   ranges    src/common/cpu_parallel.cpp:202-253 (nnz-weighted row ranges)
//   fp16/bf16 accumulate in fp32 and round once: src/common/common.h:52-79
// Compile with -ffp-contract=off so `acc += a * b` rounds the product and the
// sum separately, as the source expression reads.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <limits>
#include <stdexcept>
#include <thread>
#include <vector>

namespace {

// ---- half types ------------------------------------------------------------
struct bf16 {
  uint16_t bits;
};
inline float bf16_to_float(bf16 v) {
  uint32_t u = (uint32_t)v.bits << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
// float -> bf16, round to nearest even (NaN kept quiet).
inline bf16 float_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return bf16{(uint16_t)((u >> 16) | 0x40)};
  u += 0x7fffu + ((u >> 16) & 1u);
  return bf16{(uint16_t)(u >> 16)};
}
using f16 = _Float16;

template <typename T> struct Acc {
  static float load(T v) { return (float)v; }
  static T store(float v) { return (T)v; }
};
template <> struct Acc<bf16> {
  static float load(bf16 v) { return bf16_to_float(v); }
  static bf16 store(float v) { return float_to_bf16(v); }
};
template <typename T> bool is_zero(T v) { return Acc<T>::load(v) == 0.0f; }

// ---- nnz-weighted contiguous row ranges (cpu_parallel.cpp:184-253) ---------
struct Range {
  int64_t begin, end;
};
std::vector<Range> equal_ranges(int64_t n, int parts) {
  std::vector<Range> out;
  for (int p = 0; p < parts; ++p) {
    int64_t b = p * n / parts, e = (p + 1) * n / parts;
    if (b < e) out.push_back({b, e});
  }
  return out;
}
std::vector<Range> weighted_ranges(const std::vector<int64_t> &work, int parts) {
  const int64_t n = (int64_t)work.size();
  if (n <= 0) return {};
  if (parts <= 1) return {{0, n}};
  if (parts >= n) return equal_ranges(n, parts);
  std::vector<int64_t> prefix(n + 1, 0);
  for (int64_t i = 0; i < n; ++i) prefix[i + 1] = prefix[i] + std::max<int64_t>(0, work[i]);
  if (prefix.back() <= 0) return equal_ranges(n, parts);
  std::vector<Range> out;
  int64_t begin = 0;
  for (int part = 0; part < parts && begin < n; ++part) {
    const int remaining = parts - part;
    if (remaining == 1) {
      out.push_back({begin, n});
      break;
    }
    const int64_t rem_work = prefix.back() - prefix[begin];
    const int64_t target = prefix[begin] + (rem_work + remaining - 1) / remaining;
    int64_t end = std::lower_bound(prefix.begin() + begin + 1, prefix.end(), target) - prefix.begin();
    end = std::max(end, begin + 1);
    end = std::min(end, n - (remaining - 1));
    out.push_back({begin, end});
    begin = end;
  }
  return out;
}
template <typename Fn> void parallel_ranges(const std::vector<Range> &ranges, Fn fn) {
  if (ranges.size() <= 1) {
    for (auto &r : ranges) fn(r);
    return;
  }
  std::vector<std::thread> th;
  for (size_t i = 1; i < ranges.size(); ++i) th.emplace_back([&, i] { fn(ranges[i]); });
  fn(ranges[0]);
  for (auto &t : th) t.join();
}
template <typename I> std::vector<Range> row_ranges(const I *indptr, int64_t n_rows, int workers, int64_t scale) {
  if (workers <= 1 || n_rows <= 0) return {{0, n_rows}};
  std::vector<int64_t> work(n_rows);
  bool imbalance = false;
  for (int64_t r = 0; r < n_rows; ++r) {
    work[r] = (int64_t)(indptr[r + 1] - indptr[r]) * scale;
    if (r > 0 && work[r] != work[r - 1]) imbalance = true;
  }
  return imbalance ? weighted_ranges(work, workers) : equal_ranges(n_rows, workers);
}

// ---- SpMV -------------------------------------------------------------------
template <typename T, typename I>
void spmv(const T *data, const I *indices, const I *indptr, const T *x, T *y, int64_t n_rows, int workers) {
  auto rows = [&](Range rg) {
    for (int64_t r = rg.begin; r < rg.end; ++r) {
      float acc = 0.0f;
      for (I p = indptr[r]; p < indptr[r + 1]; ++p) acc += Acc<T>::load(data[p]) * Acc<T>::load(x[indices[p]]);
      y[r] = Acc<T>::store(acc);
    }
  };
  parallel_ranges(row_ranges(indptr, n_rows, workers, 1), rows);
}

// ---- SpMM -------------------------------------------------------------------
template <typename T, typename I>
void spmm(const T *data, const I *indices, const I *indptr, const T *rhs, int64_t k, T *out, int64_t n_rows,
          int workers) {
  auto rows = [&](Range rg) {
    std::vector<float> acc((size_t)k);
    for (int64_t r = rg.begin; r < rg.end; ++r) {
      std::fill(acc.begin(), acc.end(), 0.0f);
      for (I p = indptr[r]; p < indptr[r + 1]; ++p) {
        const float a = Acc<T>::load(data[p]);
        const T *b = rhs + (int64_t)indices[p] * k;
        for (int64_t c = 0; c < k; ++c) acc[c] += a * Acc<T>::load(b[c]);
      }
      for (int64_t c = 0; c < k; ++c) out[r * k + c] = Acc<T>::store(acc[c]);
    }
  };
  parallel_ranges(row_ranges(indptr, n_rows, workers, std::max<int64_t>(k, 1)), rows);
}

// ---- SpGEMM (Gustavson with marker + dense accumulator) ---------------------
struct SpgemmResult {
  int value_bytes = 4;
  std::vector<uint8_t> data;  // value_bytes * nnz
  std::vector<int64_t> indices;
  std::vector<int64_t> indptr;
};

void sort_touched(std::vector<int> &cols) {
  if (cols.size() <= 1) return;
  if (cols.size() <= 32) {
    for (size_t i = 1; i < cols.size(); ++i) {
      int v = cols[i];
      size_t j = i;
      while (j > 0 && v < cols[j - 1]) {
        cols[j] = cols[j - 1];
        --j;
      }
      cols[j] = v;
    }
    return;
  }
  std::sort(cols.begin(), cols.end());
}
bool dense_scan(size_t touched, int64_t dim, int disorder) {
  return touched >= 64 && dim > 0 && disorder >= 8 && (size_t)dim <= touched * 32;
}

template <typename T, typename LI, typename RI>
SpgemmResult *spgemm(const T *ld, const LI *li, const LI *lp, const T *rd, const RI *ri, const RI *rp, int64_t m,
                     int64_t rhs_rows, int64_t n) {
  auto *res = new SpgemmResult();
  res->value_bytes = sizeof(T);
  std::vector<int64_t> marker(n, -1);
  std::vector<float> accum(n, 0.0f);
  std::vector<int> cols;
  std::vector<T> out_data;
  res->indptr.assign(m + 1, 0);
  for (int64_t row = 0; row < m; ++row) {
    cols.clear();
    bool sorted = true;
    int disorder = 0;
    for (LI lpos = lp[row]; lpos < lp[row + 1]; ++lpos) {
      const int64_t rrow = (int64_t)li[lpos];
      if (rrow < 0 || rrow >= rhs_rows) throw std::invalid_argument("csr_matmat lhs indices contain an out-of-bounds column.");
      const float lv = Acc<T>::load(ld[lpos]);
      for (RI rpos = rp[rrow]; rpos < rp[rrow + 1]; ++rpos) {
        const int col = (int)ri[rpos];
        if (col < 0 || col >= n) throw std::invalid_argument("csr_matmat rhs indices contain an out-of-bounds column.");
        const float prod = lv * Acc<T>::load(rd[rpos]);
        if (marker[col] != row) {
          marker[col] = row;
          accum[col] = prod;
          if (!cols.empty() && col < cols.back()) {
            sorted = false;
            ++disorder;
          }
          cols.push_back(col);
        } else {
          accum[col] += prod;
        }
      }
    }
    auto emit = [&](int col) {
      const T v = Acc<T>::store(accum[col]);
      if (!is_zero(v)) {
        res->indices.push_back(col);
        out_data.push_back(v);
      }
    };
    if (!sorted && dense_scan(cols.size(), n, disorder)) {
      for (int64_t col = 0; col < n; ++col)
        if (marker[col] == row) emit((int)col);
    } else {
      if (!sorted) sort_touched(cols);
      for (int col : cols) emit(col);
    }
    res->indptr[row + 1] = (int64_t)out_data.size();
  }
  res->data.resize(out_data.size() * sizeof(T));
  if (!out_data.empty()) std::memcpy(res->data.data(), out_data.data(), res->data.size());
  return res;
}

// ---- CG / Jacobi PCG ----------------------------------------------------------
inline bool finite_f(float v) { return std::isfinite(v); }

template <typename I>
void spmv_f32(const float *data, const I *indices, const I *indptr, const float *x, float *out, int64_t n) {
  for (int64_t row = 0; row < n; ++row) {
    float acc = 0.0f;
    for (I p = indptr[row]; p < indptr[row + 1]; ++p) acc += data[p] * x[indices[p]];
    out[row] = acc;
  }
}
double dot_d(const std::vector<float> &a, const std::vector<float> &b) {
  double acc = 0.0;
  for (size_t i = 0; i < a.size(); ++i) acc += (double)a[i] * (double)b[i];
  return acc;
}
float dot_f(const std::vector<float> &a, const std::vector<float> &b) { return (float)dot_d(a, b); }

template <typename I>
void cg(const float *data, const I *indices, const I *indptr, const float *b, const float *x0, float *x, int64_t n,
        float rtol, float atol, int maxiter, int *info, float *residual, int *iterations) {
  std::vector<float> r(n), p(n), ap(n);
  std::copy(x0, x0 + n, x);
  spmv_f32(data, indices, indptr, x, ap.data(), n);
  double b_norm2 = 0.0, rr = 0.0;
  bool finite = true;
  for (int64_t i = 0; i < n; ++i) {
    r[i] = b[i] - ap[i];
    p[i] = r[i];
    b_norm2 += (double)b[i] * (double)b[i];
    rr += (double)r[i] * (double)r[i];
    finite = finite && finite_f(r[i]) && finite_f(p[i]) && finite_f(ap[i]) && finite_f(b[i]) && finite_f(x[i]);
  }
  const float residual_norm = (float)std::sqrt(std::max(rr, 0.0));
  const float b_norm = std::sqrt(std::max(b_norm2, 0.0));
  const float tol = std::max(atol, rtol * b_norm);
  const float eps = std::numeric_limits<float>::epsilon();
  if (!finite || !std::isfinite(rr) || !finite_f(residual_norm) || !finite_f(b_norm)) {
    *info = -3;
    *residual = residual_norm;
    *iterations = 0;
    return;
  }
  if (residual_norm <= tol) {
    *info = 0;
    *residual = residual_norm;
    *iterations = 0;
    return;
  }
  int status = maxiter > 0 ? maxiter : 1;
  int completed = 0;
  for (int it = 1; it <= maxiter; ++it) {
    spmv_f32(data, indices, indptr, p.data(), ap.data(), n);
    double denom = 0.0;
    finite = true;
    for (int64_t i = 0; i < n; ++i) {
      denom += (double)p[i] * (double)ap[i];
      finite = finite && finite_f(p[i]) && finite_f(ap[i]);
    }
    if (!finite || !std::isfinite(denom)) {
      status = -3;
      completed = it - 1;
      break;
    }
    if (std::abs(denom) <= eps) {
      double pn = 0.0, apn = 0.0;
      for (int64_t i = 0; i < n; ++i) {
        pn += (double)p[i] * (double)p[i];
        apn += (double)ap[i] * (double)ap[i];
      }
      const double scale = std::sqrt(std::max(pn * apn, 0.0));
      const double dtol = std::min((double)eps, (double)eps * (double)eps * std::max(1.0, scale));
      if (!std::isfinite(scale)) {
        status = -3;
        completed = it - 1;
        break;
      }
      if (std::abs(denom) <= dtol) {
        status = -1;
        completed = it - 1;
        break;
      }
    }
    const double alpha = rr / denom;
    if (!std::isfinite(alpha)) {
      status = -3;
      completed = it - 1;
      break;
    }
    finite = true;
    double rr_new = 0.0;
    for (int64_t i = 0; i < n; ++i) {
      const double xc = (double)x[i] + alpha * (double)p[i];
      const double rc = (double)r[i] - alpha * (double)ap[i];
      const float xf = (float)xc, rf = (float)rc;
      if (!std::isfinite(xc) || !std::isfinite(rc) || !finite_f(xf) || !finite_f(rf)) {
        finite = false;
        continue;
      }
      x[i] = xf;
      r[i] = rf;
      rr_new += (double)r[i] * (double)r[i];
    }
    const float r_norm = (float)std::sqrt(std::max(rr_new, 0.0));
    completed = it;
    if (!finite || !std::isfinite(rr_new) || !finite_f(r_norm)) {
      status = -3;
      break;
    }
    if (r_norm <= tol) {
      status = 0;
      rr = rr_new;
      break;
    }
    const double beta = rr_new / rr;
    if (!std::isfinite(beta)) {
      status = -3;
      break;
    }
    for (int64_t i = 0; i < n; ++i) {
      const double pc = (double)r[i] + beta * (double)p[i];
      const float pf = (float)pc;
      if (!std::isfinite(pc) || !finite_f(pf)) {
        status = -3;
        break;
      }
      p[i] = pf;
    }
    if (status < 0) break;
    rr = rr_new;
  }
  *info = status;
  *residual = (float)std::sqrt(std::max(rr, 0.0));
  *iterations = completed;
}

template <typename I>
void pcg_jacobi(const float *data, const I *indices, const I *indptr, const float *b, const float *x0,
                const float *inv_diag, float *x, int64_t n, float rtol, float atol, int maxiter, int *info,
                float *residual, int *iterations, int max_iters_to_run) {
  std::vector<float> r(n), z(n), p(n), ap(n);
  std::copy(x0, x0 + n, x);
  spmv_f32(data, indices, indptr, x, ap.data(), n);
  double b_norm2 = 0.0;
  bool finite = true;
  for (int64_t i = 0; i < n; ++i) {
    const float ri = b[i] - ap[i];
    const float zi = inv_diag[i] * ri;
    r[i] = ri;
    z[i] = zi;
    p[i] = zi;
    b_norm2 += (double)b[i] * (double)b[i];
    finite = finite && finite_f(ri) && finite_f(zi) && finite_f(inv_diag[i]);
  }
  float true_rr = dot_f(r, r);
  float rho = dot_f(r, z);
  const float b_norm = std::sqrt(std::max(b_norm2, 0.0));
  const float tol = std::max(atol, rtol * b_norm);
  const float true_residual = std::sqrt(std::max(true_rr, 0.0f));
  if (!finite || !finite_f(true_rr) || !finite_f(rho)) {
    *info = -3;
    *residual = true_residual;
    *iterations = 0;
    return;
  }
  if (true_residual <= tol) {
    *info = 0;
    *residual = true_residual;
    *iterations = 0;
    return;
  }
  if (rho <= 0.0f) {
    *info = -2;
    *residual = true_residual;
    *iterations = 0;
    return;
  }
  const float eps = std::numeric_limits<float>::epsilon();
  int status = maxiter > 0 ? maxiter : 1;
  int completed = 0;
  for (int it = 1; it <= maxiter; ++it) {
    if (max_iters_to_run > 0 && it > max_iters_to_run) break;  // bounded timing samples only
    spmv_f32(data, indices, indptr, p.data(), ap.data(), n);
    const float denom = dot_f(p, ap);
    const float pn = dot_f(p, p);
    const float apn = dot_f(ap, ap);
    const float scale = std::sqrt(std::max(pn * apn, 0.0f));
    const float dtol = eps * std::max(1.0f, scale);
    if (!finite_f(denom) || !finite_f(scale) || std::abs(denom) <= dtol) {
      status = -1;
      completed = it - 1;
      break;
    }
    const float alpha = rho / denom;
    if (!finite_f(alpha)) {
      status = -3;
      completed = it - 1;
      break;
    }
    double rr_acc = 0.0;
    finite = true;
    for (int64_t i = 0; i < n; ++i) {
      x[i] += alpha * p[i];
      const float ri = r[i] - alpha * ap[i];
      const float zi = inv_diag[i] * ri;
      r[i] = ri;
      z[i] = zi;
      rr_acc += (double)ri * (double)ri;
      finite = finite && finite_f(x[i]) && finite_f(ri) && finite_f(zi);
    }
    true_rr = (float)rr_acc;
    const float r_norm = std::sqrt(std::max(true_rr, 0.0f));
    completed = it;
    if (!finite || !finite_f(true_rr) || !finite_f(r_norm)) {
      status = -3;
      break;
    }
    if (r_norm <= tol) {
      status = 0;
      break;
    }
    const float rho_new = dot_f(r, z);
    if (!finite_f(rho_new) || rho_new <= 0.0f) {
      status = -2;
      break;
    }
    const float beta = rho_new / rho;
    if (!finite_f(beta)) {
      status = -3;
      break;
    }
    for (int64_t i = 0; i < n; ++i) p[i] = z[i] + beta * p[i];
    rho = rho_new;
  }
  *info = status;
  *residual = std::sqrt(std::max(true_rr, 0.0f));
  *iterations = completed;
}

// ---- COO -> CSR (src/sparse/coo_tocsr/coo_tocsr.cpp:94-237, serial path) ----
// Counting sort by row in source order, then a stable sort of every row by
// column (sort_columns) - or no sort (source order, the summation order of
// coo_matmul, src/sparse/coo_matmul/coo_matmul.cpp:~95-115).
template <typename T, typename I>
void coo_tocsr(const T *data, const I *row, const I *col, int64_t nnz, int64_t n_rows, bool sort_columns, T *out_data,
               I *out_indices, I *out_indptr, int64_t *out_perm) {
  std::fill(out_indptr, out_indptr + n_rows + 1, I{0});
  for (int64_t p = 0; p < nnz; ++p) {
    if (row[p] < 0 || (int64_t)row[p] >= n_rows) throw std::invalid_argument("coo_tocsr row out of range");
    out_indptr[(int64_t)row[p] + 1] += I{1};
  }
  for (int64_t r = 0; r < n_rows; ++r) out_indptr[r + 1] += out_indptr[r];
  std::vector<int64_t> next(out_indptr, out_indptr + n_rows), perm((size_t)nnz);
  for (int64_t p = 0; p < nnz; ++p) perm[(size_t)next[(size_t)row[p]]++] = p;
  if (sort_columns) {
    for (int64_t r = 0; r < n_rows; ++r)
      std::stable_sort(perm.begin() + (int64_t)out_indptr[r], perm.begin() + (int64_t)out_indptr[r + 1],
                       [&](int64_t a, int64_t b) { return col[a] < col[b]; });
  }
  for (int64_t q = 0; q < nnz; ++q) {
    if (out_data) out_data[q] = data[perm[(size_t)q]];
    out_indices[q] = col[perm[(size_t)q]];
    if (out_perm) out_perm[q] = perm[(size_t)q];
  }
}

// ---- COO products (src/sparse/coo_matmul/coo_matmul.cpp:~90-140) -------------
// out[row[p], :] += data[p] * rhs[col[p], :] over p in source order, fp32
// accumulation for the half types.
template <typename T, typename I>
void coo_matmul(const T *data, const I *row, const I *col, int64_t nnz, const T *rhs, int64_t k, T *out,
                int64_t n_rows) {
  std::vector<float> acc((size_t)(n_rows * k), 0.0f);
  for (int64_t p = 0; p < nnz; ++p) {
    const float a = Acc<T>::load(data[p]);
    float *o = acc.data() + (int64_t)row[p] * k;
    const T *b = rhs + (int64_t)col[p] * k;
    for (int64_t c = 0; c < k; ++c) o[c] += a * Acc<T>::load(b[c]);
  }
  for (int64_t i = 0; i < n_rows * k; ++i) out[i] = Acc<T>::store(acc[(size_t)i]);
}

// ---- transposed products (src/sparse/csr_matvec_transpose/
// csr_matvec_transpose.cpp:76-97 and csr_matmul_transpose, serial path) -------
template <typename T, typename I>
void matmul_transpose(const T *data, const I *indices, const I *indptr, int64_t n_rows, int64_t n_cols, const T *rhs,
                      int64_t k, T *out) {
  std::vector<float> acc((size_t)(n_cols * k), 0.0f);
  for (int64_t r = 0; r < n_rows; ++r)
    for (I p = indptr[r]; p < indptr[r + 1]; ++p) {
      const float a = Acc<T>::load(data[p]);
      float *o = acc.data() + (int64_t)indices[p] * k;
      for (int64_t c = 0; c < k; ++c) o[c] += a * Acc<T>::load(rhs[r * k + c]);
    }
  for (int64_t i = 0; i < n_cols * k; ++i) out[i] = Acc<T>::store(acc[(size_t)i]);
}

// ---- data cotangents (src/sparse/csr_matmul_data_vjp/
// csr_matmul_data_vjp.cpp:88-100; csr_matvec_data_vjp is the k = 1 case) ----
template <typename T, typename I>
void data_vjp(const I *indices, const I *indptr, int64_t n_rows, const T *rhs, const T *cot, int64_t k, T *out) {
  for (int64_t r = 0; r < n_rows; ++r)
    for (I p = indptr[r]; p < indptr[r + 1]; ++p) {
      float acc = 0.0f;
      for (int64_t c = 0; c < k; ++c) acc += Acc<T>::load(cot[r * k + c]) * Acc<T>::load(rhs[(int64_t)indices[p] * k + c]);
      out[p] = Acc<T>::store(acc);
    }
}

// ---- Chebyshev preconditioner and Chebyshev PCG --------------------------------
// chebyshev_apply_vector: src/preconditioners/pcg/chebyshev.cpp:84-122 (and the
// standalone apply, src/preconditioners/chebyshev/chebyshev.cpp:262-300, which
// runs the same recurrence column by column).
template <typename I>
void cheb_apply(const float *md, const I *mi, const I *mp, const float *rhs, float *out, std::vector<float> &prev,
                std::vector<float> &next, std::vector<float> &ax, int64_t n, int degree, float lmin, float lmax) {
  const float scale = 2.0f / (lmax + lmin);
  const float alpha = 1.0f - scale * lmin;
  const float mu = 1.0f / alpha;
  const float omega_prod = 2.0f / alpha;
  float c_prev = 1.0f, c_cur = mu;
  std::fill(prev.begin(), prev.end(), 0.0f);
  std::fill(next.begin(), next.end(), 0.0f);
  for (int64_t i = 0; i < n; ++i) out[i] = scale * rhs[i];
  if (degree == 1) return;
  for (int it = 1; it < degree; ++it) {
    spmv_f32(md, mi, mp, out, ax.data(), n);
    const float c_next = 2.0f * mu * c_cur - c_prev;
    const float omega = omega_prod * c_cur / c_next;
    const float one_minus_omega = 1.0f - omega;
    const float omega_scale = omega * scale;
    for (int64_t i = 0; i < n; ++i) {
      const float r = rhs[i] - ax[(size_t)i];
      next[(size_t)i] = one_minus_omega * prev[(size_t)i] + omega * out[i] + omega_scale * r;
    }
    std::copy(out, out + n, prev.begin());
    std::copy(next.begin(), next.end(), out);
    c_prev = c_cur;
    c_cur = c_next;
  }
}

// csr_pcg_chebyshev_cpu_impl: src/preconditioners/pcg/chebyshev.cpp:124-313.
template <typename I>
void pcg_chebyshev(const float *data, const I *indices, const I *indptr, const float *b, const float *x0,
                   const float *md, const I *mi, const I *mp, float *x, int64_t n, int degree, float lmin, float lmax,
                   float rtol, float atol, int maxiter, int *info, float *residual, int *iterations) {
  std::vector<float> r(n), z(n), p(n), ap(n), cp(n), cn(n), cax(n);
  std::copy(x0, x0 + n, x);
  spmv_f32(data, indices, indptr, x, ap.data(), n);
  double b_norm2 = 0.0;
  bool finite = true;
  for (int64_t i = 0; i < n; ++i) {
    const float ri = b[i] - ap[i];
    r[i] = ri;
    b_norm2 += (double)b[i] * (double)b[i];
    finite = finite && finite_f(ri) && finite_f(b[i]) && finite_f(x[i]);
  }
  cheb_apply(md, mi, mp, r.data(), z.data(), cp, cn, cax, n, degree, lmin, lmax);
  p = z;
  float true_rr = dot_f(r, r);
  float rho = dot_f(r, z);
  const float b_norm = std::sqrt(std::max(b_norm2, 0.0));
  const float tol = std::max(atol, rtol * b_norm);
  const float true_residual = std::sqrt(std::max(true_rr, 0.0f));
  if (!finite || !finite_f(true_rr) || !finite_f(rho)) {
    *info = -3; *residual = true_residual; *iterations = 0;
    return;
  }
  if (true_residual <= tol) {
    *info = 0; *residual = true_residual; *iterations = 0;
    return;
  }
  if (rho <= 0.0f) {
    *info = -2; *residual = true_residual; *iterations = 0;
    return;
  }
  const float eps = std::numeric_limits<float>::epsilon();
  int status = maxiter > 0 ? maxiter : 1;
  int completed = 0;
  for (int it = 1; it <= maxiter; ++it) {
    spmv_f32(data, indices, indptr, p.data(), ap.data(), n);
    const float denom = dot_f(p, ap);
    const float pn = dot_f(p, p);
    const float apn = dot_f(ap, ap);
    const float scale = std::sqrt(std::max(pn * apn, 0.0f));
    const float dtol = eps * std::max(1.0f, scale);
    if (!finite_f(denom) || !finite_f(scale) || std::abs(denom) <= dtol) {
      status = -1; completed = it - 1;
      break;
    }
    const float alpha = rho / denom;
    if (!finite_f(alpha)) {
      status = -3; completed = it - 1;
      break;
    }
    double rr_acc = 0.0;
    finite = true;
    for (int64_t i = 0; i < n; ++i) {
      x[i] += alpha * p[i];
      const float ri = r[i] - alpha * ap[i];
      r[i] = ri;
      rr_acc += (double)ri * (double)ri;
      finite = finite && finite_f(x[i]) && finite_f(ri);
    }
    true_rr = (float)rr_acc;
    const float r_norm = std::sqrt(std::max(true_rr, 0.0f));
    completed = it;
    if (!finite || !finite_f(true_rr) || !finite_f(r_norm)) {
      status = -3;
      break;
    }
    if (r_norm <= tol) {
      status = 0;
      break;
    }
    cheb_apply(md, mi, mp, r.data(), z.data(), cp, cn, cax, n, degree, lmin, lmax);
    const float rho_new = dot_f(r, z);
    if (!finite_f(rho_new) || rho_new <= 0.0f) {
      status = -2;
      break;
    }
    const float beta = rho_new / rho;
    if (!finite_f(beta)) {
      status = -3;
      break;
    }
    for (int64_t i = 0; i < n; ++i) p[i] = z[i] + beta * p[i];
    rho = rho_new;
  }
  *info = status;
  *residual = std::sqrt(std::max(true_rr, 0.0f));
  *iterations = completed;
}

// Gershgorin and diagonal bounds: src/preconditioners/chebyshev/chebyshev.cpp:120-161.
template <typename I>
void gershgorin(const float *data, const I *indices, const I *indptr, int64_t n_rows, float *out4) {
  double lower = std::numeric_limits<double>::infinity(), upper = -lower, dmin = lower, dmax = -lower;
  for (int64_t r = 0; r < n_rows; ++r) {
    double diag = 0.0, off = 0.0;
    for (I p = indptr[r]; p < indptr[r + 1]; ++p) {
      if ((int64_t)indices[p] == r) diag += (double)data[p];
      else off += std::abs((double)data[p]);
    }
    lower = std::min(lower, diag - off);
    upper = std::max(upper, diag + off);
    dmin = std::min(dmin, diag);
    dmax = std::max(dmax, diag);
  }
  out4[0] = (float)lower; out4[1] = (float)upper; out4[2] = (float)dmin; out4[3] = (float)dmax;
}

template <typename Fn> void by_value(int vt, Fn fn) {
  if (vt == 0) fn(float{});
  else if (vt == 1) fn(f16{});
  else if (vt == 2) fn(bf16{});
  else throw std::invalid_argument("bad value dtype");
}
template <typename Fn> void by_index(int it, Fn fn) {
  if (it == 0) fn(int32_t{});
  else if (it == 1) fn(int64_t{});
  else throw std::invalid_argument("bad index dtype");
}

thread_local char g_err[512];
template <typename Fn> int guard(Fn fn) {
  try {
    fn();
    g_err[0] = 0;
    return 0;
  } catch (const std::exception &e) {
    std::strncpy(g_err, e.what(), sizeof(g_err) - 1);
    return 1;
  }
}

}  // namespace

extern "C" {

const char *orc_last_error() { return g_err; }

int orc_csr_matvec(int vt, int it, const void *data, const void *indices, const void *indptr, const void *x,
                   void *y, int64_t n_rows, int workers) {
  return guard([&] {
    by_value(vt, [&](auto v) {
      using T = decltype(v);
      by_index(it, [&](auto i) {
        using I = decltype(i);
        spmv<T, I>((const T *)data, (const I *)indices, (const I *)indptr, (const T *)x, (T *)y, n_rows, workers);
      });
    });
  });
}

int orc_csr_matmul(int vt, int it, const void *data, const void *indices, const void *indptr, const void *rhs,
                   int64_t k, void *out, int64_t n_rows, int workers) {
  return guard([&] {
    by_value(vt, [&](auto v) {
      using T = decltype(v);
      by_index(it, [&](auto i) {
        using I = decltype(i);
        spmm<T, I>((const T *)data, (const I *)indices, (const I *)indptr, (const T *)rhs, k, (T *)out, n_rows,
                   workers);
      });
    });
  });
}

// Returns an opaque result handle (or null on error); query/copy/free below.
void *orc_csr_matmat(int vt, int lit, const void *ld, const void *li, const void *lp, int rit, const void *rd,
                     const void *ri, const void *rp, int64_t m, int64_t rhs_rows, int64_t n) {
  SpgemmResult *res = nullptr;
  int rc = guard([&] {
    by_value(vt, [&](auto v) {
      using T = decltype(v);
      by_index(lit, [&](auto a) {
        using LI = decltype(a);
        by_index(rit, [&](auto b) {
          using RI = decltype(b);
          res = spgemm<T, LI, RI>((const T *)ld, (const LI *)li, (const LI *)lp, (const T *)rd, (const RI *)ri,
                                  (const RI *)rp, m, rhs_rows, n);
        });
      });
    });
  });
  return rc == 0 ? res : nullptr;
}
int64_t orc_matmat_nnz(void *h) { return (int64_t)static_cast<SpgemmResult *>(h)->indices.size(); }
void orc_matmat_copy(void *h, void *data, int64_t *indices, int64_t *indptr) {
  auto *r = static_cast<SpgemmResult *>(h);
  if (!r->data.empty()) std::memcpy(data, r->data.data(), r->data.size());
  if (!r->indices.empty()) std::memcpy(indices, r->indices.data(), r->indices.size() * sizeof(int64_t));
  std::memcpy(indptr, r->indptr.data(), r->indptr.size() * sizeof(int64_t));
}
void orc_matmat_free(void *h) { delete static_cast<SpgemmResult *>(h); }

int orc_csr_cg(int it, const float *data, const void *indices, const void *indptr, const float *b, const float *x0,
               float *x, int64_t n, float rtol, float atol, int maxiter, int *info, float *residual,
               int *iterations) {
  return guard([&] {
    by_index(it, [&](auto i) {
      using I = decltype(i);
      cg<I>(data, (const I *)indices, (const I *)indptr, b, x0, x, n, rtol, atol, maxiter, info, residual,
            iterations);
    });
  });
}

// max_iters_to_run > 0 stops early (for bounded CPU timing samples); 0 = none.
int orc_csr_pcg_jacobi(int it, const float *data, const void *indices, const void *indptr, const float *b,
                       const float *x0, const float *inv_diag, float *x, int64_t n, float rtol, float atol,
                       int maxiter, int *info, float *residual, int *iterations, int max_iters_to_run) {
  return guard([&] {
    by_index(it, [&](auto i) {
      using I = decltype(i);
      pcg_jacobi<I>(data, (const I *)indices, (const I *)indptr, b, x0, inv_diag, x, n, rtol, atol, maxiter, info,
                    residual, iterations, max_iters_to_run);
    });
  });
}

// nnz-weighted contiguous ranges, flattened as [b0, e0, b1, e1, ...].
int orc_weighted_ranges(const int64_t *work, int64_t n, int parts, int64_t *out_pairs) {
  std::vector<int64_t> w(work, work + n);
  auto r = weighted_ranges(w, parts);
  for (size_t i = 0; i < r.size(); ++i) {
    out_pairs[2 * i] = r[i].begin;
    out_pairs[2 * i + 1] = r[i].end;
  }
  return (int)r.size();
}

int orc_coo_tocsr(int vt, int it, const void *data, const void *row, const void *col, int64_t nnz, int64_t n_rows,
                  int sort_columns, void *out_data, void *out_indices, void *out_indptr, int64_t *out_perm) {
  return guard([&] {
    by_value(vt, [&](auto v) {
      using T = decltype(v);
      by_index(it, [&](auto i) {
        using I = decltype(i);
        coo_tocsr<T, I>((const T *)data, (const I *)row, (const I *)col, nnz, n_rows, sort_columns != 0, (T *)out_data,
                        (I *)out_indices, (I *)out_indptr, out_perm);
      });
    });
  });
}

int orc_coo_matmul(int vt, int it, const void *data, const void *row, const void *col, int64_t nnz, const void *rhs,
                   int64_t k, void *out, int64_t n_rows) {
  return guard([&] {
    by_value(vt, [&](auto v) {
      using T = decltype(v);
      by_index(it, [&](auto i) {
        using I = decltype(i);
        coo_matmul<T, I>((const T *)data, (const I *)row, (const I *)col, nnz, (const T *)rhs, k, (T *)out, n_rows);
      });
    });
  });
}

int orc_csr_matmul_transpose(int vt, int it, const void *data, const void *indices, const void *indptr,
                             int64_t n_rows, int64_t n_cols, const void *rhs, int64_t k, void *out) {
  return guard([&] {
    by_value(vt, [&](auto v) {
      using T = decltype(v);
      by_index(it, [&](auto i) {
        using I = decltype(i);
        matmul_transpose<T, I>((const T *)data, (const I *)indices, (const I *)indptr, n_rows, n_cols, (const T *)rhs,
                               k, (T *)out);
      });
    });
  });
}

int orc_csr_data_vjp(int vt, int it, const void *indices, const void *indptr, int64_t n_rows, const void *rhs,
                     const void *cot, int64_t k, void *out) {
  return guard([&] {
    by_value(vt, [&](auto v) {
      using T = decltype(v);
      by_index(it, [&](auto i) {
        using I = decltype(i);
        data_vjp<T, I>((const I *)indices, (const I *)indptr, n_rows, (const T *)rhs, (const T *)cot, k, (T *)out);
      });
    });
  });
}

int orc_chebyshev_apply(int it, const float *md, const void *mi, const void *mp, int64_t n, const float *rhs,
                        int64_t k, float *out, int degree, float lmin, float lmax) {
  return guard([&] {
    by_index(it, [&](auto i) {
      using I = decltype(i);
      std::vector<float> prev(n), next(n), ax(n), col(n), res(n);
      for (int64_t c = 0; c < k; ++c) {  // column by column, as the recurrence is per column
        for (int64_t r = 0; r < n; ++r) col[r] = rhs[r * k + c];
        cheb_apply<I>(md, (const I *)mi, (const I *)mp, col.data(), res.data(), prev, next, ax, n, degree, lmin, lmax);
        for (int64_t r = 0; r < n; ++r) out[r * k + c] = res[r];
      }
    });
  });
}

int orc_csr_pcg_chebyshev(int it, const float *data, const void *indices, const void *indptr, const float *b,
                          const float *x0, const float *md, const void *mi, const void *mp, float *x, int64_t n,
                          int degree, float lmin, float lmax, float rtol, float atol, int maxiter, int *info,
                          float *residual, int *iterations) {
  return guard([&] {
    by_index(it, [&](auto i) {
      using I = decltype(i);
      pcg_chebyshev<I>(data, (const I *)indices, (const I *)indptr, b, x0, md, (const I *)mi, (const I *)mp, x, n,
                       degree, lmin, lmax, rtol, atol, maxiter, info, residual, iterations);
    });
  });
}

int orc_gershgorin(int it, const float *data, const void *indices, const void *indptr, int64_t n_rows, float *out4) {
  return guard([&] {
    by_index(it, [&](auto i) {
      using I = decltype(i);
      gershgorin<I>(data, (const I *)indices, (const I *)indptr, n_rows, out4);
    });
  });
}

}  // extern "C"
