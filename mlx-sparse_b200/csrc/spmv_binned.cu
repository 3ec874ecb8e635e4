// Builder and C-ABI front door of the row-length-binned SpMV (spmv_binned.cuh).
//
// The plan is a stable counting sort of the row ids by bin: one pass counts
// rows per (block, bin) with warp ballots, one scans the counts, one scatters
// the row ids; rows longer than the CTA bin are cut into fixed chunks on the
// host (there are few of them). Built once per matrix (the reference's CPU
// path instead recomputes nnz-weighted ranges each call,
// src/sparse/csr_matvec/csr_matvec.cpp:156-166).
#include <algorithm>
#include <vector>

#include "spmv_binned.cuh"

namespace msx {

namespace {

constexpr int kPlanThreads = 256;

__device__ __forceinline__ int bin_of(int64_t len) {
  // upper row lengths of bins 0..6 (bin 7 is everything longer)
  return len <= 8 ? 0 : len <= 16 ? 1 : len <= 32 ? 2 : len <= 64 ? 3 : len <= 128 ? 4 : len <= 512 ? 5
         : len <= 8192 ? 6 : 7;
}

template <typename I>
__global__ void __launch_bounds__(kPlanThreads)
bin_count_kernel(const I *__restrict__ indptr, int64_t n_rows, int64_t nblk, long long *__restrict__ counts,
                 unsigned long long *__restrict__ max_len) {
  __shared__ int wc[kPlanThreads / 32][kBins];
  const int64_t row = blockIdx.x * (int64_t)kPlanThreads + threadIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int bin = -1;
  int64_t len = 0;
  if (row < n_rows) {
    len = (int64_t)indptr[row + 1] - (int64_t)indptr[row];
    bin = bin_of(len);
  }
#pragma unroll
  for (int k = 0; k < kBins; ++k) {
    const unsigned m = __ballot_sync(0xffffffffu, bin == k);
    if (lane == 0) wc[warp][k] = __popc(m);
  }
  __shared__ unsigned long long wmax[kPlanThreads / 32];
  unsigned long long ml = (unsigned long long)len;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, ml, off);
    ml = o > ml ? o : ml;
  }
  if (lane == 0) wmax[warp] = ml;
  __syncthreads();
  if (threadIdx.x == 0) {  // one atomic per CTA, not per warp
    unsigned long long m = 0;
    for (int w = 0; w < kPlanThreads / 32; ++w) m = wmax[w] > m ? wmax[w] : m;
    if (m > 0) atomicMax(max_len, m);
  }
  if (threadIdx.x < kBins) {
    long long c = 0;
    for (int w = 0; w < kPlanThreads / 32; ++w) c += wc[w][threadIdx.x];
    counts[threadIdx.x * nblk + blockIdx.x] = c;
  }
}

// One CTA per bin: exclusive scan of that bin's per-block counts in place.
__global__ void __launch_bounds__(1024) bin_scan_kernel(long long *__restrict__ counts, int64_t nblk,
                                                        long long *__restrict__ totals) {
  __shared__ long long wsum[32];
  __shared__ long long chunk_total;
  long long *c = counts + blockIdx.x * nblk;
  long long carry = 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t base = 0; base < nblk; base += 1024) {
    const int64_t i = base + threadIdx.x;
    const long long v = i < nblk ? c[i] : 0;
    long long inc = v;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const long long o = __shfl_up_sync(0xffffffffu, inc, off);
      if (lane >= off) inc += o;
    }
    if (lane == 31) wsum[warp] = inc;
    __syncthreads();
    if (warp == 0) {
      long long w = wsum[lane];
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const long long o = __shfl_up_sync(0xffffffffu, w, off);
        if (lane >= off) w += o;
      }
      wsum[lane] = w;
    }
    __syncthreads();
    inc += warp > 0 ? wsum[warp - 1] : 0;
    if (i < nblk) c[i] = carry + inc - v;
    if (threadIdx.x == 1023) chunk_total = inc;
    __syncthreads();
    carry += chunk_total;
    __syncthreads();
  }
  if (threadIdx.x == 0) totals[blockIdx.x] = carry;
}

template <typename I>
__global__ void __launch_bounds__(kPlanThreads)
bin_scatter_kernel(const I *__restrict__ indptr, int64_t n_rows, int64_t nblk, const long long *__restrict__ offsets,
                   BinInfo info, int *__restrict__ rows) {
  __shared__ int wc[kPlanThreads / 32][kBins];
  const int64_t row = blockIdx.x * (int64_t)kPlanThreads + threadIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int bin = -1;
  if (row < n_rows) bin = bin_of((int64_t)indptr[row + 1] - (int64_t)indptr[row]);
  int rank = 0;
#pragma unroll
  for (int k = 0; k < kBins; ++k) {
    const unsigned m = __ballot_sync(0xffffffffu, bin == k);
    if (lane == 0) wc[warp][k] = __popc(m);
    if (bin == k) rank = __popc(m & ((1u << lane) - 1u));
  }
  __syncthreads();
  if (bin >= 0) {
    int before = 0;
    for (int w = 0; w < warp; ++w) before += wc[w][bin];
    const long long pos = info.row_start[bin] + offsets[bin * nblk + blockIdx.x] + before + rank;
    rows[pos] = (int)row;
  }
}

template <typename I>
__global__ void long_rows_kernel(const I *__restrict__ indptr, const int *__restrict__ rows, long long start,
                                 int64_t n_long, int64_t *__restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n_long) return;
  const int64_t row = rows[start + i];
  out[3 * i] = row;
  out[3 * i + 1] = (int64_t)indptr[row];
  out[3 * i + 2] = (int64_t)indptr[row + 1];
}

}  // namespace

void build_binned_plan_impl(int index_dtype, const void *indptr, int64_t n_rows, int64_t nnz, cudaStream_t s,
                            void *(*alloc)(size_t, void *), void *ctx, BinnedPlan &plan) {
  plan = BinnedPlan{};
  plan.n_rows = n_rows;
  plan.nnz = nnz;
  if (n_rows == 0) return;
  const int64_t nblk = ceil_div(n_rows, kPlanThreads);
  Scratch tmp(sizeof(long long) * (kBins * nblk + kBins) + 64, s);
  long long *counts = tmp.as<long long>();
  long long *totals = counts + kBins * nblk;
  unsigned long long *max_len = reinterpret_cast<unsigned long long *>(totals + kBins);
  MSX_CUDA(cudaMemsetAsync(max_len, 0, sizeof(unsigned long long), s));
  dispatch_index(index_dtype, [&](auto ityp) {
    using I = decltype(ityp);
    bin_count_kernel<I><<<(unsigned)nblk, kPlanThreads, 0, s>>>(static_cast<const I *>(indptr), n_rows, nblk,
                                                                counts, max_len);
  });
  bin_scan_kernel<<<kBins, 1024, 0, s>>>(counts, nblk, totals);
  MSX_CHECK_LAUNCH();
  long long h_tot[kBins + 1];
  MSX_CUDA(cudaMemcpyAsync(h_tot, totals, sizeof(long long) * (kBins + 1), cudaMemcpyDeviceToHost, s));
  MSX_CUDA(cudaStreamSynchronize(s));
  plan.max_len = (int64_t)h_tot[kBins];

  BinInfo &info = plan.info;
  int nonempty = 0, last = 0;
  long long acc = 0;
  for (int k = 0; k < kBins; ++k) {
    info.count[k] = h_tot[k];
    info.row_start[k] = acc;
    acc += h_tot[k];
    if (h_tot[k] > 0) {
      ++nonempty;
      last = k;
    }
  }
  info.identity = nonempty <= 1 ? 1 : 0;
  info.single_bin = last;
  plan.n_long = info.count[7];
  const int64_t chunks_max = plan.n_long > 0 ? plan.n_long + nnz / kLongChunk + 1 : 0;

  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const size_t rows_bytes = info.identity ? 0 : al(sizeof(int) * n_rows);
  const size_t chunk_bytes = al(sizeof(int64_t) * chunks_max);
  const size_t bytes = rows_bytes + 3 * chunk_bytes + al(sizeof(int64_t) * (plan.n_long + 1)) + 256;
  char *base = static_cast<char *>(alloc(bytes, ctx));
  plan.bytes = bytes;
  size_t off = 0;
  if (!info.identity) {
    plan.rows = reinterpret_cast<int *>(base + off);
    off += rows_bytes;
  }
  plan.chunk_row = reinterpret_cast<int64_t *>(base + off);
  off += chunk_bytes;
  plan.chunk_lo = reinterpret_cast<int64_t *>(base + off);
  off += chunk_bytes;
  plan.chunk_hi = reinterpret_cast<int64_t *>(base + off);
  off += chunk_bytes;
  plan.long_first = reinterpret_cast<int64_t *>(base + off);

  if (!info.identity) {
    dispatch_index(index_dtype, [&](auto ityp) {
      using I = decltype(ityp);
      bin_scatter_kernel<I><<<(unsigned)nblk, kPlanThreads, 0, s>>>(static_cast<const I *>(indptr), n_rows, nblk,
                                                                    counts, info, plan.rows);
    });
    MSX_CHECK_LAUNCH();
  }

  // Chunk table of the long rows (host side; there are few).
  int64_t n_chunks = 0;
  std::vector<int64_t> c_row, c_lo, c_hi, first;
  if (plan.n_long > 0) {
    Scratch lr(sizeof(int64_t) * 3 * plan.n_long, s);
    if (info.identity) {
      // every row is long: rows are 0..n-1
      std::vector<int64_t> h(3 * plan.n_long);
      std::vector<int64_t> ip(n_rows + 1);
      if (index_dtype == MSX_I32) {
        std::vector<int32_t> ip32(n_rows + 1);
        MSX_CUDA(cudaMemcpyAsync(ip32.data(), indptr, sizeof(int32_t) * (n_rows + 1), cudaMemcpyDeviceToHost, s));
        MSX_CUDA(cudaStreamSynchronize(s));
        for (int64_t r = 0; r <= n_rows; ++r) ip[r] = ip32[r];
      } else {
        MSX_CUDA(cudaMemcpyAsync(ip.data(), indptr, sizeof(int64_t) * (n_rows + 1), cudaMemcpyDeviceToHost, s));
        MSX_CUDA(cudaStreamSynchronize(s));
      }
      for (int64_t r = 0; r < n_rows; ++r) {
        h[3 * r] = r;
        h[3 * r + 1] = ip[r];
        h[3 * r + 2] = ip[r + 1];
      }
      MSX_CUDA(cudaMemcpyAsync(lr.ptr, h.data(), sizeof(int64_t) * h.size(), cudaMemcpyHostToDevice, s));
    } else {
      dispatch_index(index_dtype, [&](auto ityp) {
        using I = decltype(ityp);
        long_rows_kernel<I><<<(unsigned)ceil_div(plan.n_long, 128), 128, 0, s>>>(
            static_cast<const I *>(indptr), plan.rows, info.row_start[7], plan.n_long, lr.as<int64_t>());
      });
      MSX_CHECK_LAUNCH();
    }
    std::vector<int64_t> h(3 * plan.n_long);
    MSX_CUDA(cudaMemcpyAsync(h.data(), lr.ptr, sizeof(int64_t) * h.size(), cudaMemcpyDeviceToHost, s));
    MSX_CUDA(cudaStreamSynchronize(s));
    for (int64_t i = 0; i < plan.n_long; ++i) {
      first.push_back(n_chunks);
      for (int64_t lo = h[3 * i + 1]; lo < h[3 * i + 2]; lo += kLongChunk) {
        c_row.push_back(h[3 * i]);
        c_lo.push_back(lo);
        c_hi.push_back(std::min<int64_t>(lo + kLongChunk, h[3 * i + 2]));
        ++n_chunks;
      }
    }
    first.push_back(n_chunks);
    MSX_CUDA(cudaMemcpyAsync(plan.chunk_row, c_row.data(), sizeof(int64_t) * n_chunks, cudaMemcpyHostToDevice, s));
    MSX_CUDA(cudaMemcpyAsync(plan.chunk_lo, c_lo.data(), sizeof(int64_t) * n_chunks, cudaMemcpyHostToDevice, s));
    MSX_CUDA(cudaMemcpyAsync(plan.chunk_hi, c_hi.data(), sizeof(int64_t) * n_chunks, cudaMemcpyHostToDevice, s));
    MSX_CUDA(cudaMemcpyAsync(plan.long_first, first.data(), sizeof(int64_t) * first.size(), cudaMemcpyHostToDevice,
                             s));
    MSX_CUDA(cudaStreamSynchronize(s));  // host vectors go out of scope
  }
  plan.n_chunks = n_chunks;

  long long blocks = 0;
  for (int k = 0; k < kBins; ++k) {
    info.block_start[k] = blocks;
    if (k <= 5) blocks += ceil_div((int64_t)info.count[k] << k, kBinThreads);
    else if (k == 6) blocks += info.count[6];
    else blocks += n_chunks;
  }
  info.block_start[kBins] = blocks;
  MSX_CUDA(cudaStreamSynchronize(s));
}

void spmv_binned_run(int value_dtype, int index_dtype, const BinnedPlan &plan, const void *data, const void *indices,
                     const void *indptr, const void *x, void *y, float *carry, cudaStream_t stream) {
  dispatch_value(value_dtype, [&](auto vtyp) {
    using T = decltype(vtyp);
    dispatch_index(index_dtype, [&](auto ityp) {
      using I = decltype(ityp);
      launch_spmv_binned<T, I, NoEpilogue>(plan, static_cast<const T *>(data), static_cast<const I *>(indices),
                                      static_cast<const I *>(indptr), static_cast<const T *>(x), static_cast<T *>(y),
                                      carry, NoEpilogue{}, stream);
      launch_spmv_long_fixup<T>(plan, carry, static_cast<T *>(y), stream);
    });
  });
}

}  // namespace msx
