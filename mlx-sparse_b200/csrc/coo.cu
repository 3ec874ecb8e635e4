// COO -> CSR conversion, CSR transposition and the data cotangents of the
// products, for sm_100a.
//
// Reference behaviour:
//  - coo_tocsr (src/sparse/coo_tocsr/coo_tocsr.cpp:94-237): entries are
//    counted per row, scattered to their row in source order (a stable
//    counting sort), then every row is stably sorted by column. Duplicates
//    stay, in source order. The result is sorted by (row, column, source
//    position).
//  - coo_matmul (src/sparse/coo_matmul/coo_matmul.cpp:~95-140) sums every
//    output row over its entries in source order; a CSR copy whose rows keep
//    the source order ("stored order" below) reproduces that order exactly.
//  - csr_matvec_transpose / csr_matmul_transpose (src/sparse/
//    csr_matvec_transpose/csr_matvec_transpose.cpp:76-97): out[col] sums
//    data[p] * x[row] over the nonzeros in row-major order. The transposed
//    CSR built here lists each column's entries in that same order, so a
//    plain SpMV / SpMM over it sums in the reference's order.
//  - csr_matvec_data_vjp / csr_matmul_data_vjp (src/sparse/
//    csr_matmul_data_vjp/csr_matmul_data_vjp.cpp:88-100): out[p] =
//    cot[row] * x[col], or the dot of cot[row, :] and B[col, :] summed over
//    k in order, fp32-accumulated.
//
// B200 design. The conversion is integer and byte work bound by HBM: a
// histogram with atomics, the device scan, a scatter with per-row atomic
// cursors (which loses the source order), then a segmented sort that restores
// a unique order because every key carries its source position: rows of <= 32
// entries are insertion-sorted by one thread, rows of <= 2048 by a CTA with a
// bitonic network in shared memory, longer rows by one CTA each with chunk
// sorts and merge passes in global memory. The result is therefore exactly
// the reference's, whatever order the atomics took.
#include <climits>

#include "common.cuh"
#include "ops.cuh"
#include "scan.cuh"

namespace msx {

namespace {

constexpr int kSortThreads = 256;
constexpr int kThreadSortMax = 32;   // rows up to this length: one thread
constexpr int kCtaSortMax = 2048;    // up to this: one CTA, shared memory

struct SortKey {
  long long k;  // column (or 0 when sorting by source position only)
  long long p;  // source position
};

__device__ __forceinline__ bool key_less(const SortKey &a, const SortKey &b) {
  return a.k < b.k || (a.k == b.k && a.p < b.p);
}

template <typename I>
__device__ __forceinline__ SortKey make_key(const I *__restrict__ col, long long p, bool by_col) {
  return SortKey{by_col ? (long long)col[p] : 0ll, p};
}

template <typename I>
__global__ void coo_hist_kernel(const I *__restrict__ row, const I *__restrict__ col, int64_t nnz, int64_t n_rows,
                                int64_t n_cols, unsigned long long *__restrict__ cnt, int *__restrict__ flags) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < nnz; p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = (int64_t)row[p], c = (int64_t)col[p];
    if (r < 0 || r >= n_rows || c < 0 || c >= n_cols) {
      atomicOr(&flags[0], 1);
    } else {
      atomicAdd(&cnt[r], 1ull);
    }
  }
}

template <typename I>
__global__ void copy_indptr_kernel(const int64_t *__restrict__ src, int64_t n, I *__restrict__ dst) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = (I)src[i];
}

template <typename I>
__global__ void coo_scatter_kernel(const I *__restrict__ row, int64_t nnz, int64_t n_rows,
                                   unsigned long long *__restrict__ cursor, long long *__restrict__ perm) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < nnz; p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = (int64_t)row[p];
    if (r < 0 || r >= n_rows) continue;  // flagged by the histogram
    const unsigned long long dst = atomicAdd(&cursor[r], 1ull);
    perm[dst] = p;
  }
}

// One thread per row: sorts rows of <= kThreadSortMax entries in place and
// lists the longer ones for the CTA kernels.
template <typename I>
__global__ void short_sort_kernel(const I *__restrict__ indptr, int64_t n_rows, const I *__restrict__ col,
                                  bool by_col, long long *__restrict__ perm, long long *__restrict__ med_rows,
                                  long long *__restrict__ long_rows, int *__restrict__ flags) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < n_rows;
       r += (int64_t)gridDim.x * blockDim.x) {
    const int64_t start = (int64_t)indptr[r];
    const int64_t len = (int64_t)indptr[r + 1] - start;
    if (len <= 1) continue;
    if (len > kThreadSortMax) {
      if (len <= kCtaSortMax) med_rows[atomicAdd(&flags[1], 1)] = r;
      else long_rows[atomicAdd(&flags[2], 1)] = r;
      continue;
    }
    SortKey a[kThreadSortMax];
    for (int j = 0; j < len; ++j) a[j] = make_key(col, perm[start + j], by_col);
    for (int j = 1; j < len; ++j) {
      const SortKey v = a[j];
      int i = j - 1;
      while (i >= 0 && key_less(v, a[i])) {
        a[i + 1] = a[i];
        --i;
      }
      a[i + 1] = v;
    }
    for (int j = 0; j < len; ++j) perm[start + j] = a[j].p;
  }
}

// Bitonic sort of `len` (a power of two) keys in shared memory by the CTA.
__device__ void cta_bitonic(SortKey *key, int len) {
  for (int k = 2; k <= len; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < len; i += blockDim.x) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const SortKey a = key[i], b = key[ixj];
          const bool up = (i & k) == 0;
          if (key_less(b, a) == up) {
            key[i] = b;
            key[ixj] = a;
          }
        }
      }
      __syncthreads();
    }
  }
}

// Sorts perm[start, start + len) (len <= kCtaSortMax) with the CTA.
template <typename I>
__device__ void cta_sort_range(long long *__restrict__ perm, int64_t start, int len, const I *__restrict__ col,
                               bool by_col, SortKey *sh) {
  int pw = 1;
  while (pw < len) pw <<= 1;
  for (int j = threadIdx.x; j < pw; j += blockDim.x)
    sh[j] = j < len ? make_key(col, perm[start + j], by_col) : SortKey{LLONG_MAX, LLONG_MAX};
  __syncthreads();
  cta_bitonic(sh, pw);
  for (int j = threadIdx.x; j < len; j += blockDim.x) perm[start + j] = sh[j].p;
  __syncthreads();
}

template <typename I>
__global__ void __launch_bounds__(kSortThreads)
medium_sort_kernel(const I *__restrict__ indptr, const long long *__restrict__ rows, const I *__restrict__ col,
                   bool by_col, long long *__restrict__ perm) {
  __shared__ SortKey sh[kCtaSortMax];
  const int64_t r = rows[blockIdx.x];
  const int64_t start = (int64_t)indptr[r];
  cta_sort_range(perm, start, (int)((int64_t)indptr[r + 1] - start), col, by_col, sh);
}

// Number of entries of the sorted run src[lo, hi) whose key is below `key`.
template <typename I>
__device__ __forceinline__ int64_t rank_in_run(const long long *__restrict__ src, int64_t lo, int64_t hi,
                                               const SortKey &key, const I *__restrict__ col, bool by_col) {
  int64_t a = lo, b = hi;
  while (a < b) {
    const int64_t m = (a + b) >> 1;
    if (key_less(make_key(col, src[m], by_col), key)) a = m + 1;
    else b = m;
  }
  return a - lo;
}

// One CTA per row longer than kCtaSortMax: chunk sorts in shared memory, then
// merge passes between perm and tmp (same offsets); the result ends in perm.
template <typename I>
__global__ void __launch_bounds__(kSortThreads)
long_sort_kernel(const I *__restrict__ indptr, const long long *__restrict__ rows, const I *__restrict__ col,
                 bool by_col, long long *__restrict__ perm, long long *__restrict__ tmp) {
  __shared__ SortKey sh[kCtaSortMax];
  const int64_t r = rows[blockIdx.x];
  const int64_t start = (int64_t)indptr[r];
  const int64_t len = (int64_t)indptr[r + 1] - start;
  for (int64_t c = 0; c < len; c += kCtaSortMax)
    cta_sort_range(perm, start + c, (int)min((int64_t)kCtaSortMax, len - c), col, by_col, sh);
  long long *src = perm + start, *dst = tmp + start;
  for (int64_t w = kCtaSortMax; w < len; w <<= 1) {
    for (int64_t i = threadIdx.x; i < len; i += blockDim.x) {
      const int64_t lb = (i / (2 * w)) * (2 * w);
      const int64_t mid = min(lb + w, len), hi = min(lb + 2 * w, len);
      const SortKey key = make_key(col, src[i], by_col);
      const int64_t pos = i < mid ? (i - lb) + rank_in_run(src, mid, hi, key, col, by_col)
                                  : (i - mid) + rank_in_run(src, lb, mid, key, col, by_col);
      dst[lb + pos] = src[i];
    }
    __syncthreads();
    long long *t = src;
    src = dst;
    dst = t;
  }
  if (src != perm + start) {
    for (int64_t i = threadIdx.x; i < len; i += blockDim.x) perm[start + i] = src[i];
  }
}

template <typename T, typename I>
__global__ void gather_kernel(const long long *__restrict__ perm, int64_t nnz, const T *__restrict__ data,
                              const I *__restrict__ col, T *__restrict__ out_data, I *__restrict__ out_idx,
                              long long *__restrict__ out_perm) {
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < nnz; q += (int64_t)gridDim.x * blockDim.x) {
    const long long p = perm[q];
    if (out_data) out_data[q] = data[p];
    out_idx[q] = col[p];
    if (out_perm) out_perm[q] = p;
  }
}

template <typename I>
__global__ void expand_rows_kernel(const I *__restrict__ indptr, int64_t n_rows, I *__restrict__ rowid) {
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < n_rows;
       r += (int64_t)gridDim.x * blockDim.x)
    for (int64_t p = (int64_t)indptr[r]; p < (int64_t)indptr[r + 1]; ++p) rowid[p] = (I)r;
}

int stream_grid(int64_t n, int threads = 256) {
  const int64_t cap = (int64_t)num_sms() * 8;
  const int64_t g = ceil_div(std::max<int64_t>(n, 1), threads);
  return (int)(g < cap ? g : cap);
}

}  // namespace

void coo_tocsr_run(int value_dtype, int index_dtype, const void *data, const void *row, const void *col, int64_t nnz,
                   int64_t n_rows, int64_t n_cols, bool by_col, void *out_data, void *out_indices, void *out_indptr,
                   int64_t *out_perm, cudaStream_t s) {
  dispatch_index(index_dtype, [&](auto ityp) {
    using I = decltype(ityp);
    I *oip = static_cast<I *>(out_indptr);
    if (nnz == 0 || n_rows == 0) {
      if (nnz > 0) fail(MSX_ERR_INVALID, "coo_tocsr row index out of range for a matrix with no rows.");
      MSX_CUDA(cudaMemsetAsync(oip, 0, sizeof(I) * (size_t)(n_rows + 1), s));
      return;
    }
    const I *ro = static_cast<const I *>(row);
    const I *co = static_cast<const I *>(col);
    const int64_t n_sums = scan_scratch_elems(n_rows);
    const int64_t list_cap = std::min<int64_t>(n_rows, nnz / (kThreadSortMax + 1) + 1);
    auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
    size_t off = 0;
    const size_t o_cnt = off; off += al(sizeof(int64_t) * n_rows);
    const size_t o_cur = off; off += al(sizeof(int64_t) * (n_rows + 1));
    const size_t o_sums = off; off += al(sizeof(int64_t) * n_sums);
    const size_t o_perm = off; off += al(sizeof(long long) * nnz);
    const size_t o_med = off; off += al(sizeof(long long) * list_cap);
    const size_t o_long = off; off += al(sizeof(long long) * list_cap);
    const size_t o_flags = off; off += al(sizeof(int) * 4);
    Scratch scratch(off, s);
    char *base = scratch.as<char>();
    auto *cnt = reinterpret_cast<int64_t *>(base + o_cnt);
    auto *cursor = reinterpret_cast<int64_t *>(base + o_cur);
    auto *sums = reinterpret_cast<int64_t *>(base + o_sums);
    auto *perm = reinterpret_cast<long long *>(base + o_perm);
    auto *med = reinterpret_cast<long long *>(base + o_med);
    auto *lng = reinterpret_cast<long long *>(base + o_long);
    auto *flags = reinterpret_cast<int *>(base + o_flags);
    MSX_CUDA(cudaMemsetAsync(cnt, 0, sizeof(int64_t) * n_rows, s));
    MSX_CUDA(cudaMemsetAsync(flags, 0, sizeof(int) * 4, s));
    coo_hist_kernel<I><<<stream_grid(nnz), 256, 0, s>>>(ro, co, nnz, n_rows, n_cols,
                                                        reinterpret_cast<unsigned long long *>(cnt), flags);
    MSX_CHECK_LAUNCH();
    scan_counts_to_indptr<int64_t>(cnt, n_rows, cursor, sums, s);
    copy_indptr_kernel<I><<<stream_grid(n_rows + 1), 256, 0, s>>>(cursor, n_rows + 1, oip);
    coo_scatter_kernel<I><<<stream_grid(nnz), 256, 0, s>>>(ro, nnz, n_rows,
                                                           reinterpret_cast<unsigned long long *>(cursor), perm);
    short_sort_kernel<I><<<stream_grid(n_rows, 128), 128, 0, s>>>(oip, n_rows, co, by_col, perm, med, lng, flags);
    MSX_CHECK_LAUNCH();
    int host_flags[4] = {0, 0, 0, 0};
    MSX_CUDA(cudaMemcpyAsync(host_flags, flags, sizeof(host_flags), cudaMemcpyDeviceToHost, s));
    MSX_CUDA(cudaStreamSynchronize(s));
    if (host_flags[0]) fail(MSX_ERR_INVALID, "coo_tocsr coordinates must lie inside the matrix shape.");
    if (host_flags[1] > 0) {
      medium_sort_kernel<I><<<host_flags[1], kSortThreads, 0, s>>>(oip, med, co, by_col, perm);
      MSX_CHECK_LAUNCH();
    }
    if (host_flags[2] > 0) {
      Scratch tmp(sizeof(long long) * nnz, s);
      long_sort_kernel<I><<<host_flags[2], kSortThreads, 0, s>>>(oip, lng, co, by_col, perm, tmp.as<long long>());
      MSX_CHECK_LAUNCH();
    }
    if (out_data) {
      dispatch_value(value_dtype, [&](auto vtyp) {
        using T = decltype(vtyp);
        gather_kernel<T, I><<<stream_grid(nnz), 256, 0, s>>>(perm, nnz, static_cast<const T *>(data), co,
                                                             static_cast<T *>(out_data), static_cast<I *>(out_indices),
                                                             reinterpret_cast<long long *>(out_perm));
      });
    } else {
      gather_kernel<float, I><<<stream_grid(nnz), 256, 0, s>>>(perm, nnz, nullptr, co, nullptr,
                                                               static_cast<I *>(out_indices),
                                                               reinterpret_cast<long long *>(out_perm));
    }
    MSX_CHECK_LAUNCH();
  });
}

void csr_transpose_run(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
                       int64_t nnz, int64_t n_rows, int64_t n_cols, void *out_data, void *out_indices,
                       void *out_indptr, int64_t *out_perm, cudaStream_t s) {
  dispatch_index(index_dtype, [&](auto ityp) {
    using I = decltype(ityp);
    Scratch rowid(sizeof(I) * (size_t)std::max<int64_t>(nnz, 1), s);
    if (nnz > 0) {
      expand_rows_kernel<I><<<stream_grid(n_rows, 128), 128, 0, s>>>(static_cast<const I *>(indptr), n_rows,
                                                                      rowid.as<I>());
      MSX_CHECK_LAUNCH();
    }
    // the columns become rows; each keeps its entries in row-major source
    // order, i.e. by ascending original row
    coo_tocsr_run(value_dtype, index_dtype, data, indices, rowid.as<I>(), nnz, n_cols, n_rows, false, out_data,
                  out_indices, out_indptr, out_perm, s);
  });
}

// ---- data cotangents ---------------------------------------------------------
namespace {

constexpr int kVjpThreads = 256;
constexpr int kVjpPerCta = 1024;  // nonzeros per CTA

// Row of nonzero p: the last r in [lo, hi] with indptr[r] <= p.
template <typename I>
__device__ __forceinline__ int64_t row_of(const I *__restrict__ indptr, int64_t lo, int64_t hi, int64_t p) {
  while (lo < hi) {
    const int64_t m = (lo + hi + 1) >> 1;
    if ((int64_t)indptr[m] <= p) lo = m;
    else hi = m - 1;
  }
  return lo;
}

template <typename T, typename I>
__global__ void __launch_bounds__(kVjpThreads)
data_vjp_kernel(const I *__restrict__ indices, const I *__restrict__ indptr, int64_t nnz, int64_t n_rows,
                const T *__restrict__ rhs, const T *__restrict__ cot, int64_t k, T *__restrict__ out) {
  __shared__ int64_t bounds[2];
  const int64_t p0 = blockIdx.x * (int64_t)kVjpPerCta;
  const int64_t p1 = min(p0 + (int64_t)kVjpPerCta, nnz);
  if (threadIdx.x < 2) bounds[threadIdx.x] = row_of(indptr, 0, n_rows - 1, threadIdx.x == 0 ? p0 : p1 - 1);
  __syncthreads();
  const int64_t rlo = bounds[0], rhi = bounds[1];
  for (int64_t p = p0 + threadIdx.x; p < p1; p += kVjpThreads) {
    const int64_t r = row_of(indptr, rlo, rhi, p);
    const int64_t c = (int64_t)indices[p];
    const T *a = cot + r * k;
    const T *b = rhs + c * k;
    float acc = 0.f;
    for (int64_t j = 0; j < k; ++j) acc = add_rn(acc, mul_rn(VT<T>::load(a[j]), VT<T>::load(b[j])));
    out[p] = VT<T>::store(acc);
  }
}

}  // namespace

void csr_data_vjp_run(int value_dtype, int index_dtype, const void *indices, const void *indptr, int64_t nnz,
                      int64_t n_rows, const void *rhs, const void *cot, int64_t k, void *out, cudaStream_t s) {
  if (nnz == 0) return;
  dispatch_value(value_dtype, [&](auto vtyp) {
    using T = decltype(vtyp);
    dispatch_index(index_dtype, [&](auto ityp) {
      using I = decltype(ityp);
      if (k == 0) {
        MSX_CUDA(cudaMemsetAsync(out, 0, sizeof(T) * (size_t)nnz, s));
        return;
      }
      data_vjp_kernel<T, I><<<(unsigned)ceil_div(nnz, kVjpPerCta), kVjpThreads, 0, s>>>(
          static_cast<const I *>(indices), static_cast<const I *>(indptr), nnz, n_rows, static_cast<const T *>(rhs),
          static_cast<const T *>(cot), k, static_cast<T *>(out));
      MSX_CHECK_LAUNCH();
    });
  });
}

}  // namespace msx
