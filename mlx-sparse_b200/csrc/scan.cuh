// Exclusive scan of per-row counts into a CSR row pointer (device-wide,
// three launches: block sums, one-CTA scan of the block sums, block scans
// with the carried offsets). Shared by SpGEMM and the COO conversion.
#pragma once
#include "common.cuh"

namespace msx {
namespace {

// ---- scan of row counts into indptr ----------------------------------------------
constexpr int kScanThreads = 1024;

__device__ __forceinline__ int64_t block_inclusive_scan(int64_t v, int64_t *smem) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int64_t o = __shfl_up_sync(0xffffffffu, v, off);
    if (lane >= off) v += o;
  }
  if (lane == 31) smem[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int64_t w = lane < (kScanThreads / 32) ? smem[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int64_t o = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += o;
    }
    smem[lane] = w;
  }
  __syncthreads();
  const int64_t add = warp > 0 ? smem[warp - 1] : 0;
  __syncthreads();
  return v + add;
}

__global__ void __launch_bounds__(kScanThreads)
scan_block_sums(const int64_t *__restrict__ in, int64_t m, int64_t *__restrict__ sums) {
  __shared__ int64_t smem[32];
  const int64_t i = blockIdx.x * (int64_t)kScanThreads + threadIdx.x;
  const int64_t v = i < m ? in[i] : 0;
  const int64_t inc = block_inclusive_scan(v, smem);
  if (threadIdx.x == kScanThreads - 1) sums[blockIdx.x] = inc;
}

__global__ void __launch_bounds__(kScanThreads)
scan_sums_serial(int64_t *__restrict__ sums, int64_t nb, int64_t *__restrict__ total) {
  __shared__ int64_t smem[32];
  __shared__ int64_t chunk_total;
  int64_t carry = 0;
  for (int64_t base = 0; base < nb; base += kScanThreads) {
    const int64_t i = base + threadIdx.x;
    const int64_t v = i < nb ? sums[i] : 0;
    const int64_t inc = block_inclusive_scan(v, smem);
    if (i < nb) sums[i] = carry + inc - v;  // exclusive offsets of the blocks
    if (threadIdx.x == kScanThreads - 1) chunk_total = inc;
    __syncthreads();
    carry += chunk_total;
    __syncthreads();
  }
  if (threadIdx.x == 0) *total = carry;
}

template <typename OutI>
__global__ void __launch_bounds__(kScanThreads)
scan_write_indptr(const int64_t *__restrict__ in, int64_t m, const int64_t *__restrict__ sums,
                  OutI *__restrict__ indptr) {
  __shared__ int64_t smem[32];
  const int64_t i = blockIdx.x * (int64_t)kScanThreads + threadIdx.x;
  const int64_t v = i < m ? in[i] : 0;
  const int64_t inc = block_inclusive_scan(v, smem) + sums[blockIdx.x];
  if (i < m) indptr[i + 1] = (OutI)inc;
  if (i == 0) indptr[0] = 0;
}

}  // namespace

// int64 scratch the scan needs for m counts; the total lands in the last one.
inline int64_t scan_scratch_elems(int64_t m) { return ceil_div(m, kScanThreads) + 1; }

// indptr[0] = 0, indptr[i + 1] = counts[0] + ... + counts[i]; the total is
// left in sums[scan_scratch_elems(m) - 1] (device). m must be > 0.
template <typename OutI>
void scan_counts_to_indptr(const int64_t *counts, int64_t m, OutI *indptr, int64_t *sums, cudaStream_t s) {
  const int64_t nb = ceil_div(m, kScanThreads);
  scan_block_sums<<<(unsigned)nb, kScanThreads, 0, s>>>(counts, m, sums);
  scan_sums_serial<<<1, kScanThreads, 0, s>>>(sums, nb, sums + nb);
  scan_write_indptr<OutI><<<(unsigned)nb, kScanThreads, 0, s>>>(counts, m, sums, indptr);
  MSX_CHECK_LAUNCH();
}

}  // namespace msx
