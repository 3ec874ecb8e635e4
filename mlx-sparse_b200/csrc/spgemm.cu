// CSR x CSR (SpGEMM) -> canonical CSR for sm_100a.
//
// Reference behaviour: src/sparse/csr_matmat/csr_matmat.cpp:544-650 (Gustavson
// with a marker array and a dense accumulator): for output row i, the products
// a[i,k] * b[k,j] are visited in lhs-position then rhs-position order; the first
// product of a column initialises its accumulator (fp32 for fp16/bf16 values),
// later ones are added; the row is emitted in ascending column order and an
// entry is dropped when its value, rounded to the storage type, is exactly
// zero (:613-641). Output index dtype: the inputs' when both agree, else int64
// (:1354-1356); nnz must fit int32 and the index dtype (:478-488).
//
// B200 design: two passes (symbolic count, numeric fill) over rows binned by
// their product count W:
//   W <= 256     one warp per row: expand the W products into shared memory
//                with 64-bit keys (column << 32 | position), bitonic-sort them,
//                then sum each column's run in position order - the reference's
//                exact accumulation order - and compact with warp ballots;
//   W <= 4096    the same with one CTA per row;
//   W  > 4096    one CTA per row over a dense global accumulator (marker +
//                value per column): lhs entries are applied one after another,
//                the entries of one rhs row in parallel (rhs rows without
//                repeated columns) or by one thread (otherwise), then columns
//                are extracted in ascending order.
// The symbolic pass computes the exact pruned counts (it must evaluate the
// values to know which cancel), a device scan builds indptr, and the numeric
// pass writes each row at its offset. No atomics touch values, so results are
// deterministic.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "scan.cuh"

namespace msx {

namespace {

constexpr int kWarpCap = 256;    // products per warp-level row
constexpr int kBlockCap = 4096;  // products per CTA-level row
constexpr int kBlockThreads = 256;
constexpr int kDenseThreads = 512;

__device__ __forceinline__ uint32_t key_col(uint64_t k) { return (uint32_t)(k >> 32); }
__device__ __forceinline__ uint32_t key_seq(uint64_t k) { return (uint32_t)(k & 0xffffffffu); }

// ---- row work and binning ------------------------------------------------------
template <typename LI, typename RI>
__global__ void row_work_kernel(const LI *__restrict__ li, const LI *__restrict__ lp, const RI *__restrict__ rp,
                                int64_t m, int64_t rhs_rows, int64_t *__restrict__ work, int *__restrict__ err) {
  const int64_t row = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (row >= m) return;
  int64_t w = 0;
  for (int64_t q = (int64_t)lp[row]; q < (int64_t)lp[row + 1]; ++q) {
    const int64_t k = (int64_t)li[q];
    if (k < 0 || k >= rhs_rows) {
      atomicOr(err, 1);
      continue;
    }
    w += (int64_t)rp[k + 1] - (int64_t)rp[k];
  }
  work[row] = w;
}

// Flags rhs rows whose columns are out of range (bit 2) or not strictly
// increasing (bit 4: repeated columns possible).
template <typename RI>
__global__ void rhs_check_kernel(const RI *__restrict__ ri, const RI *__restrict__ rp, int64_t rhs_rows,
                                 int64_t n_cols, int *__restrict__ err) {
  const int64_t row = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (row >= rhs_rows) return;
  int64_t prev = -1;
  int flags = 0;
  for (int64_t q = (int64_t)rp[row]; q < (int64_t)rp[row + 1]; ++q) {
    const int64_t c = (int64_t)ri[q];
    if (c < 0 || c >= n_cols) flags |= 2;
    if (c <= prev) flags |= 4;
    prev = c;
  }
  if (flags) atomicOr(err, flags);
}

__global__ void bin_kernel(const int64_t *__restrict__ work, int64_t m, int *__restrict__ lists,
                           int *__restrict__ counts, int64_t *__restrict__ row_nnz) {
  const int64_t row = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (row >= m) return;
  const int64_t w = work[row];
  int bin;
  if (w == 0) {
    if (row_nnz) row_nnz[row] = 0;
    return;
  } else if (w <= kWarpCap) {
    bin = 0;
  } else if (w <= kBlockCap) {
    bin = 1;
  } else {
    bin = 2;
  }
  const int slot = atomicAdd(counts + bin, 1);
  lists[bin * m + slot] = (int)row;
}

// ---- expand / sort / compress ---------------------------------------------------
// Sorts `len` (power of two) keys in shared memory with `nthreads` threads
// starting at `tid`; `sync` is a barrier over those threads.
template <typename Sync>
__device__ __forceinline__ void bitonic_sort(uint64_t *key, int len, int tid, int nthreads, Sync sync) {
  for (int k = 2; k <= len; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < len; i += nthreads) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const uint64_t a = key[i], b = key[ixj];
          const bool up = (i & k) == 0;
          if ((a > b) == up) {
            key[i] = b;
            key[ixj] = a;
          }
        }
      }
      sync();
    }
  }
}

template <typename T, typename LI, typename RI, typename OutI, bool kWrite, int kCap, bool kWarp>
struct EscRow {
  // Processes one row with `nthreads` cooperating threads (a warp or a CTA).
  __device__ static void run(int64_t row, int tid, int nthreads, uint64_t *key, float *val, int *scratch_cnt,
                             const T *__restrict__ ld, const LI *__restrict__ li, const LI *__restrict__ lp,
                             const T *__restrict__ rd, const RI *__restrict__ ri, const RI *__restrict__ rp,
                             const OutI *__restrict__ out_indptr, OutI *__restrict__ out_idx,
                             T *__restrict__ out_data, int64_t *__restrict__ row_nnz, bool prune) {
    auto sync = [&]() {
      if (kWarp) __syncwarp();
      else __syncthreads();
    };
    // expand in (lhs position, rhs position) order
    int cnt = 0;
    for (int64_t q = (int64_t)lp[row]; q < (int64_t)lp[row + 1]; ++q) {
      const int64_t k = (int64_t)li[q];
      const float lv = VT<T>::load(ld[q]);
      const int64_t rb = (int64_t)rp[k];
      const int len = (int)((int64_t)rp[k + 1] - rb);
      for (int j = tid; j < len; j += nthreads) {
        const int s = cnt + j;
        key[s] = ((uint64_t)(uint32_t)ri[rb + j] << 32) | (uint32_t)s;
        val[s] = __fmul_rn(lv, VT<T>::load(rd[rb + j]));
      }
      cnt += len;
    }
    int pw = 1;
    while (pw < cnt) pw <<= 1;
    for (int j = cnt + tid; j < pw; j += nthreads) key[j] = ~0ull;
    sync();
    bitonic_sort(key, pw, tid, nthreads, sync);
    // sum runs in position order and compact
    const int64_t out0 = kWrite ? (int64_t)out_indptr[row] : 0;
    int count = 0;
    const int lane = tid & 31;
    const int warp = tid >> 5;
    const int nwarps = (nthreads + 31) >> 5;
    for (int base = 0; base < cnt; base += nthreads) {
      const int j = base + tid;
      bool keep = false;
      uint32_t col = 0;
      T out_v{};
      if (j < cnt) {
        col = key_col(key[j]);
        const bool head = (j == 0) || key_col(key[j - 1]) != col;
        if (head) {
          float s = val[key_seq(key[j])];
          for (int t = j + 1; t < cnt && key_col(key[t]) == col; ++t) s = __fadd_rn(s, val[key_seq(key[t])]);
          out_v = VT<T>::store(s);
          keep = !prune || VT<T>::load(out_v) != 0.0f;
        }
      }
      const unsigned mask = __ballot_sync(0xffffffffu, keep);
      int pos;
      if (kWarp) {
        pos = count + __popc(mask & ((1u << lane) - 1u));
        count += __popc(mask);
      } else {
        // block-wide exclusive count over warps in order
        if (lane == 0) scratch_cnt[warp] = __popc(mask);
        __syncthreads();
        int before = 0, total = 0;
        for (int w = 0; w < nwarps; ++w) {
          const int c = scratch_cnt[w];
          if (w < warp) before += c;
          total += c;
        }
        pos = count + before + __popc(mask & ((1u << lane) - 1u));
        count += total;
        __syncthreads();
      }
      if (kWrite && keep) {
        out_idx[out0 + pos] = (OutI)col;
        out_data[out0 + pos] = out_v;
      }
    }
    if (!kWrite && tid == 0) row_nnz[row] = count;
    sync();
  }
};

template <typename T, typename LI, typename RI, typename OutI, bool kWrite>
__global__ void __launch_bounds__(kBlockThreads)
spgemm_warp_kernel(const int *__restrict__ list, const int *__restrict__ count_ptr, const T *__restrict__ ld,
                   const LI *__restrict__ li, const LI *__restrict__ lp, const T *__restrict__ rd,
                   const RI *__restrict__ ri, const RI *__restrict__ rp, const OutI *__restrict__ out_indptr,
                   OutI *__restrict__ out_idx, T *__restrict__ out_data, int64_t *__restrict__ row_nnz, bool prune) {
  __shared__ uint64_t keys[kBlockThreads / 32][kWarpCap];
  __shared__ float vals[kBlockThreads / 32][kWarpCap];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int count = *count_ptr;
  for (int w = blockIdx.x * (kBlockThreads / 32) + warp; w < count; w += gridDim.x * (kBlockThreads / 32)) {
    EscRow<T, LI, RI, OutI, kWrite, kWarpCap, true>::run(list[w], lane, 32, keys[warp], vals[warp], nullptr, ld, li,
                                                         lp, rd, ri, rp, out_indptr, out_idx, out_data, row_nnz,
                                                         prune);
  }
}

template <typename T, typename LI, typename RI, typename OutI, bool kWrite>
__global__ void __launch_bounds__(kBlockThreads)
spgemm_block_kernel(const int *__restrict__ list, const int *__restrict__ count_ptr, const T *__restrict__ ld,
                    const LI *__restrict__ li, const LI *__restrict__ lp, const T *__restrict__ rd,
                    const RI *__restrict__ ri, const RI *__restrict__ rp, const OutI *__restrict__ out_indptr,
                    OutI *__restrict__ out_idx, T *__restrict__ out_data, int64_t *__restrict__ row_nnz,
                    bool prune) {
  extern __shared__ __align__(16) unsigned char dyn[];
  uint64_t *keys = reinterpret_cast<uint64_t *>(dyn);
  float *vals = reinterpret_cast<float *>(keys + kBlockCap);
  __shared__ int cnt[kBlockThreads / 32];
  const int count = *count_ptr;
  for (int b = blockIdx.x; b < count; b += gridDim.x) {
    EscRow<T, LI, RI, OutI, kWrite, kBlockCap, false>::run(list[b], threadIdx.x, kBlockThreads, keys, vals, cnt,
                                                           ld, li, lp, rd, ri, rp, out_indptr, out_idx, out_data,
                                                           row_nnz, prune);
  }
}

// Rows with more than kBlockCap products: dense per-CTA accumulator slot.
template <typename T, typename LI, typename RI, typename OutI, bool kWrite>
__global__ void __launch_bounds__(kDenseThreads)
spgemm_dense_kernel(const int *__restrict__ list, const int *__restrict__ count_ptr, const T *__restrict__ ld,
                    const LI *__restrict__ li, const LI *__restrict__ lp, const T *__restrict__ rd,
                    const RI *__restrict__ ri, const RI *__restrict__ rp, int64_t n_cols,
                    int *__restrict__ marker_base, float *__restrict__ accum_base, const int *__restrict__ flags,
                    const OutI *__restrict__ out_indptr, OutI *__restrict__ out_idx, T *__restrict__ out_data,
                    int64_t *__restrict__ row_nnz, bool prune) {
  __shared__ int wcnt[kDenseThreads / 32];
  int *marker = marker_base + (int64_t)blockIdx.x * n_cols;
  float *accum = accum_base + (int64_t)blockIdx.x * n_cols;
  const bool parallel_rhs = ((*flags) & 4) == 0;  // rhs rows have no repeated columns
  const int count = *count_ptr;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int b = blockIdx.x; b < count; b += gridDim.x) {
    const int row = list[b];
    for (int64_t q = (int64_t)lp[row]; q < (int64_t)lp[row + 1]; ++q) {
      const int64_t k = (int64_t)li[q];
      const float lv = VT<T>::load(ld[q]);
      const int64_t rb = (int64_t)rp[k], re = (int64_t)rp[k + 1];
      if (parallel_rhs) {
        for (int64_t j = rb + tid; j < re; j += kDenseThreads) {
          const int64_t c = (int64_t)ri[j];
          const float prod = __fmul_rn(lv, VT<T>::load(rd[j]));
          if (marker[c] != row) {
            marker[c] = row;
            accum[c] = prod;
          } else {
            accum[c] = __fadd_rn(accum[c], prod);
          }
        }
      } else if (tid == 0) {
        for (int64_t j = rb; j < re; ++j) {
          const int64_t c = (int64_t)ri[j];
          const float prod = __fmul_rn(lv, VT<T>::load(rd[j]));
          if (marker[c] != row) {
            marker[c] = row;
            accum[c] = prod;
          } else {
            accum[c] = __fadd_rn(accum[c], prod);
          }
        }
      }
      __syncthreads();
    }
    // ordered extraction
    const int64_t out0 = kWrite ? (int64_t)out_indptr[row] : 0;
    int64_t written = 0;
    for (int64_t base = 0; base < n_cols; base += kDenseThreads) {
      const int64_t c = base + tid;
      bool keep = false;
      T v{};
      if (c < n_cols && marker[c] == row) {
        v = VT<T>::store(accum[c]);
        keep = !prune || VT<T>::load(v) != 0.0f;
      }
      const unsigned mask = __ballot_sync(0xffffffffu, keep);
      if (lane == 0) wcnt[warp] = __popc(mask);
      __syncthreads();
      int before = 0, total = 0;
      for (int w = 0; w < kDenseThreads / 32; ++w) {
        if (w < warp) before += wcnt[w];
        total += wcnt[w];
      }
      if (kWrite && keep) {
        const int64_t pos = out0 + written + before + __popc(mask & ((1u << lane) - 1u));
        out_idx[pos] = (OutI)c;
        out_data[pos] = v;
      }
      written += total;
      __syncthreads();
    }
    if (!kWrite && tid == 0) row_nnz[row] = written;
    __syncthreads();
  }
}

struct Bins {
  int counts[3];
};

int dense_slots(int64_t n_cols) {
  const int64_t budget = (int64_t)256 << 20;
  int64_t slots = budget / std::max<int64_t>(n_cols * 8, 1);
  slots = std::max<int64_t>(1, std::min<int64_t>(slots, 2 * num_sms()));
  return (int)slots;
}

template <typename T, typename LI, typename RI, typename OutI>
void spgemm_pass(bool write, const T *ld, const LI *li, const LI *lp, const T *rd, const RI *ri, const RI *rp,
                 int64_t m, int64_t rhs_rows, int64_t n_cols, OutI *out_indptr, OutI *out_idx, T *out_data,
                 int64_t *out_nnz, bool prune, cudaStream_t s) {
  if (m == 0) {
    if (!write) {
      OutI zero = 0;
      MSX_CUDA(cudaMemcpyAsync(out_indptr, &zero, sizeof(OutI), cudaMemcpyHostToDevice, s));
      MSX_CUDA(cudaStreamSynchronize(s));
      *out_nnz = 0;
    }
    return;
  }
  const int slots = dense_slots(n_cols);
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const int64_t nb = ceil_div(m, kScanThreads);
  size_t off = 0;
  const size_t o_work = off; off += al(sizeof(int64_t) * m);
  const size_t o_rownnz = off; off += al(sizeof(int64_t) * m);
  const size_t o_lists = off; off += al(sizeof(int) * 3 * m);
  const size_t o_counts = off; off += al(sizeof(int) * 8);
  const size_t o_sums = off; off += al(sizeof(int64_t) * (nb + 1));
  const size_t o_marker = off; off += al(sizeof(int) * (size_t)slots * n_cols);
  const size_t o_accum = off; off += al(sizeof(float) * (size_t)slots * n_cols);
  Scratch scratch(off, s);
  char *base = scratch.as<char>();
  int64_t *work = reinterpret_cast<int64_t *>(base + o_work);
  int64_t *row_nnz = reinterpret_cast<int64_t *>(base + o_rownnz);
  int *lists = reinterpret_cast<int *>(base + o_lists);
  int *counts = reinterpret_cast<int *>(base + o_counts);  // [0..2] bins, [3] flags
  int64_t *sums = reinterpret_cast<int64_t *>(base + o_sums);
  int *marker = reinterpret_cast<int *>(base + o_marker);
  float *accum = reinterpret_cast<float *>(base + o_accum);
  int *flags = counts + 3;

  MSX_CUDA(cudaMemsetAsync(counts, 0, sizeof(int) * 8, s));
  const int t = 256;
  row_work_kernel<LI, RI><<<(unsigned)ceil_div(m, t), t, 0, s>>>(li, lp, rp, m, rhs_rows, work, flags);
  if (rhs_rows > 0)
    rhs_check_kernel<RI><<<(unsigned)ceil_div(rhs_rows, t), t, 0, s>>>(ri, rp, rhs_rows, n_cols, flags);
  bin_kernel<<<(unsigned)ceil_div(m, t), t, 0, s>>>(work, m, lists, counts, row_nnz);
  MSX_CHECK_LAUNCH();
  int host_counts[4];
  MSX_CUDA(cudaMemcpyAsync(host_counts, counts, sizeof(host_counts), cudaMemcpyDeviceToHost, s));
  MSX_CUDA(cudaStreamSynchronize(s));
  if (host_counts[3] & 1) fail(MSX_ERR_INVALID, "csr_matmat lhs indices contain an out-of-bounds column.");
  if (host_counts[3] & 2) fail(MSX_ERR_INVALID, "csr_matmat rhs indices contain an out-of-bounds column.");

  const int sms = num_sms();
  if (host_counts[0] > 0) {
    const int warps_per_block = kBlockThreads / 32;
    const int grid = (int)std::min<int64_t>(ceil_div(host_counts[0], warps_per_block), (int64_t)sms * 8);
    if (write)
      spgemm_warp_kernel<T, LI, RI, OutI, true><<<grid, kBlockThreads, 0, s>>>(
          lists, counts + 0, ld, li, lp, rd, ri, rp, out_indptr, out_idx, out_data, row_nnz, prune);
    else
      spgemm_warp_kernel<T, LI, RI, OutI, false><<<grid, kBlockThreads, 0, s>>>(
          lists, counts + 0, ld, li, lp, rd, ri, rp, out_indptr, out_idx, out_data, row_nnz, prune);
    MSX_CHECK_LAUNCH();
  }
  if (host_counts[1] > 0) {
    const size_t smem = (size_t)kBlockCap * (sizeof(uint64_t) + sizeof(float));
    const int grid = (int)std::min<int64_t>(host_counts[1], (int64_t)sms * 4);
    if (write) {
      auto kern = spgemm_block_kernel<T, LI, RI, OutI, true>;
      MSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      kern<<<grid, kBlockThreads, smem, s>>>(lists + m, counts + 1, ld, li, lp, rd, ri, rp, out_indptr, out_idx,
                                             out_data, row_nnz, prune);
    } else {
      auto kern = spgemm_block_kernel<T, LI, RI, OutI, false>;
      MSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      kern<<<grid, kBlockThreads, smem, s>>>(lists + m, counts + 1, ld, li, lp, rd, ri, rp, out_indptr, out_idx,
                                             out_data, row_nnz, prune);
    }
    MSX_CHECK_LAUNCH();
  }
  if (host_counts[2] > 0) {
    MSX_CUDA(cudaMemsetAsync(marker, 0xff, sizeof(int) * (size_t)slots * n_cols, s));
    const int grid = std::min(host_counts[2], slots);
    if (write)
      spgemm_dense_kernel<T, LI, RI, OutI, true><<<grid, kDenseThreads, 0, s>>>(
          lists + 2 * m, counts + 2, ld, li, lp, rd, ri, rp, n_cols, marker, accum, flags, out_indptr, out_idx,
          out_data, row_nnz, prune);
    else
      spgemm_dense_kernel<T, LI, RI, OutI, false><<<grid, kDenseThreads, 0, s>>>(
          lists + 2 * m, counts + 2, ld, li, lp, rd, ri, rp, n_cols, marker, accum, flags, out_indptr, out_idx,
          out_data, row_nnz, prune);
    MSX_CHECK_LAUNCH();
  }
  if (write) return;

  scan_counts_to_indptr<OutI>(row_nnz, m, out_indptr, sums, s);
  int64_t total = 0;
  MSX_CUDA(cudaMemcpyAsync(&total, sums + nb, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
  MSX_CUDA(cudaStreamSynchronize(s));
  if (total > (int64_t)INT32_MAX) fail(MSX_ERR_OVERFLOW, "csr_matmat output nnz exceeds MLX shape limits.");
  if (sizeof(OutI) == 4 && total > (int64_t)INT32_MAX)
    fail(MSX_ERR_OVERFLOW, "csr_matmat output nnz exceeds index dtype capacity.");
  *out_nnz = total;
}

}  // namespace

void spgemm_run(bool write, int value_dtype, int lhs_it, const void *ld, const void *li, const void *lp, int rhs_it,
                const void *rd, const void *ri, const void *rp, int64_t m, int64_t rhs_rows, int64_t n_cols,
                int out_it, void *out_indptr, void *out_idx, void *out_data, int64_t *out_nnz, bool prune,
                cudaStream_t s) {
  dispatch_value(value_dtype, [&](auto vt) {
    using T = decltype(vt);
    dispatch_index(lhs_it, [&](auto a) {
      using LI = decltype(a);
      dispatch_index(rhs_it, [&](auto b) {
        using RI = decltype(b);
        dispatch_index(out_it, [&](auto c) {
          using OutI = decltype(c);
          spgemm_pass<T, LI, RI, OutI>(write, static_cast<const T *>(ld), static_cast<const LI *>(li),
                                       static_cast<const LI *>(lp), static_cast<const T *>(rd),
                                       static_cast<const RI *>(ri), static_cast<const RI *>(rp), m, rhs_rows,
                                       n_cols, static_cast<OutI *>(out_indptr), static_cast<OutI *>(out_idx),
                                       static_cast<T *>(out_data), out_nnz, prune, s);
        });
      });
    });
  });
}

}  // namespace msx
