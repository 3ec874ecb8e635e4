// Row-length-binned CSR SpMV (the planned path).
//
// Rows are sorted (stably, once per matrix) into bins by their length; one
// launch serves every bin with a block range of its own:
//   bin 0  len <= 8      1 lane per row (the row is summed sequentially, in the
//                        reference's order; all 8 loads of a row in flight)
//   bin 1  len <= 16     2 lanes per row
//   bin 2  len <= 32     4 lanes
//   bin 3  len <= 64     8 lanes
//   bin 4  len <= 128    16 lanes
//   bin 5  len <= 512    a warp per row
//   bin 6  len <= 8192   a CTA per row
//   bin 7  longer        8192-nonzero chunks, one CTA each; chunk partials are
//                        added in chunk order by a small fixup kernel.
// Within a bin rows keep ascending order; when a single bin holds every row the
// row list is the identity and is not stored. Lanes of a group stride over the
// row (coalesced within the group) and their partials are combined by a
// shuffle tree, so results are deterministic.
#pragma once
#include <vector>

#include "common.cuh"

namespace msx {

constexpr int kBins = 8;
constexpr int kBinThreads = 256;
constexpr int kLongChunk = 8192;

struct BinInfo {
  long long block_start[kBins + 1];  // cumulative block counts per bin
  long long row_start[kBins];        // offset of the bin in the row list
  long long count[kBins];            // rows per bin
  int identity;                      // 1: the row list is 0..n-1 (not stored)
  int single_bin;                    // bin holding every row when identity
};

// Device buffers of a binned plan (one allocation).
struct BinnedPlan {
  BinInfo info{};
  int64_t n_rows = 0, nnz = 0;
  int *rows = nullptr;             // row list (n_rows) unless identity
  int64_t n_chunks = 0;            // bin-7 chunks
  int64_t n_long = 0;              // bin-7 rows
  int64_t *chunk_row = nullptr;    // per chunk: row
  int64_t *chunk_lo = nullptr;     // per chunk: first nonzero
  int64_t *chunk_hi = nullptr;     // per chunk: end nonzero
  int64_t *long_first = nullptr;   // per long row: first chunk (n_long + 1)
  int64_t max_len = 0;
  size_t bytes = 0;
};

// Builds the plan; `alloc` returns device memory of the requested size that
// outlives the plan's use. Synchronises `stream`.
template <typename Alloc>
void build_binned_plan(int index_dtype, const void *indptr, int64_t n_rows, int64_t nnz, cudaStream_t stream,
                       Alloc alloc, BinnedPlan &plan);
void build_binned_plan_impl(int index_dtype, const void *indptr, int64_t n_rows, int64_t nnz, cudaStream_t stream,
                            void *(*alloc)(size_t, void *), void *ctx, BinnedPlan &plan);
template <typename Alloc>
void build_binned_plan(int index_dtype, const void *indptr, int64_t n_rows, int64_t nnz, cudaStream_t stream,
                       Alloc alloc, BinnedPlan &plan) {
  build_binned_plan_impl(
      index_dtype, indptr, n_rows, nnz, stream,
      [](size_t b, void *c) -> void * { return (*static_cast<Alloc *>(c))(b); }, &alloc, plan);
}

// Carry buffer (floats) the long-row chunks need: plan.n_chunks.

template <typename T>
__device__ __forceinline__ float group_sum(float v, int G) {
  for (int off = G >> 1; off > 0; off >>= 1) v = add_rn(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

template <typename T, typename I, typename Epi>
__global__ void __launch_bounds__(kBinThreads, 4)  // 64 registers, no spills: 4 CTAs/SM instead of 3
spmv_binned_kernel(const T *__restrict__ data, const I *__restrict__ indices, const I *__restrict__ indptr,
                   const T *__restrict__ x, T *__restrict__ y, const int *__restrict__ rows, BinInfo info,
                   const int64_t *__restrict__ chunk_row, const int64_t *__restrict__ chunk_lo,
                   const int64_t *__restrict__ chunk_hi, float *__restrict__ carry, Epi epi) {
  __shared__ float red[kBinThreads / 32];
  pdl_wait();
  pdl_trigger();
  if (epi.skip()) return;
  for (long long b = blockIdx.x; b < info.block_start[kBins]; b += gridDim.x) {
  int bin = 0;
#pragma unroll
  for (int k = 1; k < kBins; ++k)
    if (b >= info.block_start[k]) bin = k;
  const long long lb = b - info.block_start[bin];
  const int tid = threadIdx.x;
  if (bin <= 5) {
    const int G = 1 << bin;
    const long long group = (lb * kBinThreads + tid) >> bin;
    const int lane_g = tid & (G - 1);
    const bool active = group < info.count[bin];
    int64_t row = 0;
    float acc = 0.f;
    if (active) {
      const long long pos = info.row_start[bin] + group;
      row = info.identity ? pos : (int64_t)rows[pos];
      const int64_t p0 = (int64_t)__ldg(indptr + row), p1 = (int64_t)__ldg(indptr + row + 1);
      if (G == 1) {
        // <= 8 nonzeros: issue every load of the row at once, then sum in order
        I c[8];
        T v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (p0 + u < p1) {
            c[u] = ld_stream(indices + p0 + u);
            v[u] = ld_stream(data + p0 + u);
          }
        }
        float xv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (p0 + u < p1) xv[u] = VT<T>::load(__ldg(x + c[u]));
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (p0 + u < p1) acc = add_rn(acc, mul_rn(VT<T>::load(v[u]), xv[u]));
      } else {
        int64_t p = p0 + lane_g;
        for (; p + 3 * G < p1; p += 4 * G) {
          I c[4];
          T v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            c[u] = ld_stream(indices + p + u * G);
            v[u] = ld_stream(data + p + u * G);
          }
          float xv[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) xv[u] = VT<T>::load(__ldg(x + c[u]));
#pragma unroll
          for (int u = 0; u < 4; ++u) acc = add_rn(acc, mul_rn(VT<T>::load(v[u]), xv[u]));
        }
        for (; p < p1; p += G) acc = add_rn(acc, mul_rn(VT<T>::load(ld_stream(data + p)),
                                                        VT<T>::load(__ldg(x + ld_stream(indices + p)))));
      }
    }
    if (G > 1) acc = group_sum<T>(acc, G);
    if (active && lane_g == 0) {
      const T out = VT<T>::store(acc);
      y[row] = out;
      epi.row(row, VT<T>::load(out));
    }
  } else {
    int64_t row, p0, p1;
    if (bin == 6) {
      row = info.identity ? info.row_start[6] + lb : (int64_t)rows[info.row_start[6] + lb];
      p0 = (int64_t)__ldg(indptr + row);
      p1 = (int64_t)__ldg(indptr + row + 1);
    } else {
      row = chunk_row[lb];
      p0 = chunk_lo[lb];
      p1 = chunk_hi[lb];
    }
    float acc = 0.f;
    int64_t p = p0 + tid;
    for (; p + 3 * kBinThreads < p1; p += 4 * kBinThreads) {
      I c[4];
      T v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        c[u] = ld_stream(indices + p + u * kBinThreads);
        v[u] = ld_stream(data + p + u * kBinThreads);
      }
      float xv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) xv[u] = VT<T>::load(__ldg(x + c[u]));
#pragma unroll
      for (int u = 0; u < 4; ++u) acc = add_rn(acc, mul_rn(VT<T>::load(v[u]), xv[u]));
    }
    for (; p < p1; p += kBinThreads)
      acc = add_rn(acc, mul_rn(VT<T>::load(ld_stream(data + p)), VT<T>::load(__ldg(x + ld_stream(indices + p)))));
    acc = group_sum<T>(acc, 32);
    if ((tid & 31) == 0) red[tid >> 5] = acc;
    __syncthreads();
    if (tid == 0) {
      float s = red[0];
#pragma unroll
      for (int w = 1; w < kBinThreads / 32; ++w) s = add_rn(s, red[w]);
      if (bin == 6) {
        const T out = VT<T>::store(s);
        y[row] = out;
        epi.row(row, VT<T>::load(out));
      } else {
        carry[lb] = s;
      }
    }
    __syncthreads();  // red[] is reused by the next virtual block
  }
  }
  epi.finish();
}

// Long rows: y[row] = sum of its chunk partials in chunk order.
template <typename T>
__global__ void spmv_long_fixup_kernel(const int *__restrict__ rows, BinInfo info, const int64_t *__restrict__ first,
                                       const float *__restrict__ carry, T *__restrict__ y, int64_t n_long) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n_long) return;
  const long long pos = info.row_start[7] + i;
  const int64_t row = info.identity ? pos : (int64_t)rows[pos];
  float s = carry[first[i]];
  for (int64_t c = first[i] + 1; c < first[i + 1]; ++c) s = add_rn(s, carry[c]);
  y[row] = VT<T>::store(s);
}

// ---- consecutive short rows -----------------------------------------------------
// Every row has at most 8 nonzeros and the row list is the identity (stencil
// matrices such as the 2D Laplacian and 3D Poisson operators). A CTA takes 256
// consecutive rows: it copies their row offsets and then their contiguous
// nonzero range into shared memory with cp.async (16-byte copies of the range's
// aligned window - 4x fewer copy instructions than per-element copies - so the
// loads in flight hold no registers and 8 CTAs fit an SM), then each thread
// sums its row left to right - the reference's order - with every x gather of
// the row issued at once.
__device__ __forceinline__ void cp_async_4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_8(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <typename V>
__device__ __forceinline__ void stage_elem(V *dst, const V *src) {
  if constexpr (sizeof(V) == 8) cp_async_8(dst, src);
  else if constexpr (sizeof(V) == 4) cp_async_4(dst, src);
  else *dst = ld_stream(src);
}

constexpr int kShortRowsPerBlock = 256;

__device__ __forceinline__ void cp_async_16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

// Stages elements [k0, k0 + K) of `src` (an array of `total` elements) into
// shared memory `dst` (16-byte aligned, room for K + 16 / sizeof(V) - 1
// elements) with 16-byte cp.async copies: the copied window starts at the
// 16-byte boundary at or below k0, so element k0 + e lands at
// dst[e + shift]; returns shift. Chunks that would read past the array's end
// (or start before its beginning) are copied element by element.
template <typename V>
__device__ __forceinline__ int stage_range16(V *dst, const V *src, int64_t k0, int K, int64_t total, int tid,
                                             int nthreads) {
  constexpr int kPer = 16 / (int)sizeof(V);
  const int shift = (int)(((reinterpret_cast<uintptr_t>(src + k0)) & 15u) / sizeof(V));
  const int64_t w0 = k0 - shift;  // first element of the window (16-byte aligned)
  const int chunks = (shift + K + kPer - 1) / kPer;
  for (int c = tid; c < chunks; c += nthreads) {
    const int64_t g = w0 + (int64_t)c * kPer;
    if (g >= 0 && g + kPer <= total) {
      cp_async_16(dst + c * kPer, src + g);
    } else {  // the window would start before the array or end past it
      for (int u = 0; u < kPer; ++u)
        if (g + u >= k0 && g + u < k0 + K) stage_elem(dst + c * kPer + u, src + g + u);
    }
  }
  return shift;
}

template <typename T, typename I, typename Epi>
__global__ void __launch_bounds__(kShortRowsPerBlock, Epi::kMinBlocks)
spmv_short_kernel(const T *__restrict__ data, const I *__restrict__ indices, const I *__restrict__ indptr,
                  const T *__restrict__ x, T *__restrict__ y, int64_t n_rows, int64_t nnz, Epi epi) {
  __shared__ I ptr_s[kShortRowsPerBlock + 1];
  __shared__ __align__(16) I idx_s[kShortRowsPerBlock * 8 + 16 / sizeof(I)];
  __shared__ __align__(16) T val_s[kShortRowsPerBlock * 8 + 16 / sizeof(T)];
  pdl_wait();
  pdl_trigger();
  if (epi.skip()) return;
  const int64_t halo_from = epi.halo_from();  // multi-GPU: halo columns come from the epilogue
  const int tid = threadIdx.x;
  const int64_t nblk = (n_rows + kShortRowsPerBlock - 1) / kShortRowsPerBlock;
  for (int64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
    const int64_t r0 = blk * kShortRowsPerBlock;
    const int nr = (int)min((int64_t)kShortRowsPerBlock, n_rows - r0);
    if (tid < nr) stage_elem(&ptr_s[tid], indptr + r0 + tid);
    if (tid == 0) stage_elem(&ptr_s[nr], indptr + r0 + nr);
    cp_async_wait_all();
    __syncthreads();
    const int64_t k0 = (int64_t)ptr_s[0];
    const int K = (int)((int64_t)ptr_s[nr] - k0);
    const int si = stage_range16(idx_s, indices, k0, K, nnz, tid, kShortRowsPerBlock);
    const int sv = stage_range16(val_s, data, k0, K, nnz, tid, kShortRowsPerBlock);
    cp_async_wait_all();
    __syncthreads();
    if (tid < nr) {
      const int q0 = (int)((int64_t)ptr_s[tid] - k0);
      const int q1 = (int)((int64_t)ptr_s[tid + 1] - k0);
      float xv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (q0 + u < q1) {
          const I c = idx_s[si + q0 + u];
          if constexpr (Epi::kHalo)
            xv[u] = (int64_t)c >= halo_from ? epi.halo_x(c) : VT<T>::load(__ldg(x + c));
          else
            xv[u] = VT<T>::load(__ldg(x + c));
        }
      float acc = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (q0 + u < q1) acc = add_rn(acc, mul_rn(VT<T>::load(val_s[sv + q0 + u]), xv[u]));
      const T out = VT<T>::store(acc);
      y[r0 + tid] = out;
      epi.row(r0 + tid, VT<T>::load(out));
    }
    __syncthreads();  // shared arrays are refilled for the next block
  }
  epi.finish();
}

// Pipelined variant for small matrices (few row blocks per CTA, where the
// three dependent round trips of each block - offsets, nonzeros, x - dominate):
// while block j is summed from shared memory, block j+1's nonzeros and block
// j+2's row offsets are already in flight (cp.async groups). Three offset
// buffers and two nonzero buffers in dynamic shared memory.
template <typename I>
constexpr size_t short_ptr_bytes() {
  return ((3 * (kShortRowsPerBlock + 1) * sizeof(I)) + 15) & ~size_t(15);
}
// nonzero buffers hold a block's range plus the alignment shift (one 16-byte chunk)
template <typename V>
constexpr int kShortBufElems = kShortRowsPerBlock * 8 + 16 / (int)sizeof(V);
template <typename T, typename I>
constexpr size_t short_pipe_smem_bytes() {
  return short_ptr_bytes<I>() + 2 * (size_t)kShortBufElems<I> * sizeof(I) + 2 * (size_t)kShortBufElems<T> * sizeof(T);
}

template <typename T, typename I, typename Epi>
__global__ void __launch_bounds__(kShortRowsPerBlock)
spmv_short_pipe_kernel(const T *__restrict__ data, const I *__restrict__ indices, const I *__restrict__ indptr,
                       const T *__restrict__ x, T *__restrict__ y, int64_t n_rows, int64_t nnz, Epi epi) {
  extern __shared__ __align__(16) unsigned char short_smem[];
  using PtrBuf = I[kShortRowsPerBlock + 1];
  constexpr int kIdxElems = kShortRowsPerBlock * 8 + 16 / (int)sizeof(I);
  constexpr int kValElems = kShortRowsPerBlock * 8 + 16 / (int)sizeof(T);
  PtrBuf *ptr_s = reinterpret_cast<PtrBuf *>(short_smem);
  I *idx_base = reinterpret_cast<I *>(short_smem + short_ptr_bytes<I>());
  T *val_base = reinterpret_cast<T *>(short_smem + short_ptr_bytes<I>() + 2 * sizeof(I) * kIdxElems);
  pdl_wait();
  pdl_trigger();
  if (epi.skip()) return;
  const int64_t halo_from = epi.halo_from();
  const int tid = threadIdx.x;
  const int64_t nblk = (n_rows + kShortRowsPerBlock - 1) / kShortRowsPerBlock;
  auto rows_of = [&](int64_t blk) { return (int)min((int64_t)kShortRowsPerBlock, n_rows - blk * kShortRowsPerBlock); };
  auto load_ptr = [&](int64_t blk, int buf) {
    if (blk >= nblk) return;
    const int64_t r0 = blk * kShortRowsPerBlock;
    const int nr = rows_of(blk);
    if (tid < nr) stage_elem(&ptr_s[buf][tid], indptr + r0 + tid);
    if (tid == 0) stage_elem(&ptr_s[buf][nr], indptr + r0 + nr);
  };
  auto load_data = [&](int64_t blk, int pbuf, int dbuf) {
    if (blk >= nblk) return;
    const int nr = rows_of(blk);
    const int64_t k0 = (int64_t)ptr_s[pbuf][0];
    const int K = (int)((int64_t)ptr_s[pbuf][nr] - k0);
    stage_range16(idx_base + dbuf * kIdxElems, indices, k0, K, nnz, tid, kShortRowsPerBlock);
    stage_range16(val_base + dbuf * kValElems, data, k0, K, nnz, tid, kShortRowsPerBlock);
  };
  const int64_t G = gridDim.x;
  int64_t blk = blockIdx.x;
  load_ptr(blk, 0);
  cp_async_wait_all();
  __syncthreads();
  load_data(blk, 0, 0);
  load_ptr(blk + G, 1);
  for (int j = 0; blk < nblk; ++j, blk += G) {
    const int pc = j % 3, pn = (j + 1) % 3, pnn = (j + 2) % 3, dc = j & 1, dn = dc ^ 1;
    cp_async_wait_all();
    __syncthreads();  // block j's nonzeros and block j+1's offsets have landed
    load_data(blk + G, pn, dn);
    load_ptr(blk + 2 * G, pnn);
    const int64_t r0 = blk * kShortRowsPerBlock;
    const int nr = rows_of(blk);
    if (tid < nr) {
      const int64_t k0 = (int64_t)ptr_s[pc][0];
      // the same alignment shifts stage_range16 used for this block
      const int si = (int)(((reinterpret_cast<uintptr_t>(indices + k0)) & 15u) / sizeof(I));
      const int sv = (int)(((reinterpret_cast<uintptr_t>(data + k0)) & 15u) / sizeof(T));
      const int q0 = (int)((int64_t)ptr_s[pc][tid] - k0);
      const int q1 = (int)((int64_t)ptr_s[pc][tid + 1] - k0);
      float xv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (q0 + u < q1) {
          const I c = idx_base[dc * kIdxElems + si + q0 + u];
          if constexpr (Epi::kHalo)
            xv[u] = (int64_t)c >= halo_from ? epi.halo_x(c) : VT<T>::load(__ldg(x + c));
          else
            xv[u] = VT<T>::load(__ldg(x + c));
        }
      float acc = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (q0 + u < q1) acc = add_rn(acc, mul_rn(VT<T>::load(val_base[dc * kValElems + sv + q0 + u]), xv[u]));
      const T out = VT<T>::store(acc);
      y[r0 + tid] = out;
      epi.row(r0 + tid, VT<T>::load(out));
    }
    __syncthreads();  // buffers of block j are refilled two steps later
  }
  cp_async_wait_all();
  epi.finish();
}

inline bool short_rows_plan(const BinnedPlan &plan) { return plan.info.identity && plan.info.single_bin == 0; }

// Grid and kernel choice of the short-row path: the single-stage kernel on a
// persistent grid, or the pipelined kernel when that grid would give each CTA
// at most kShortPipeMaxBlocks row blocks or the epilogue asks for it
// (Epi::kShortPipe; MSX_SPMV_SHORT_PIPE=0/1 forces either).
constexpr int64_t kShortPipeMaxBlocks = 8;
struct ShortLaunch {
  bool pipe;
  int64_t grid;
};

template <typename T, typename I, typename Epi>
ShortLaunch short_launch(int64_t n_rows) {
  static thread_local int cached_dev = -1, per_sm = 0, per_sm_pipe = 0, sms = 0, force = -1;
  int dev = 0;
  MSX_CUDA(cudaGetDevice(&dev));
  if (dev != cached_dev) {
    int occ = 0;
    MSX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmv_short_kernel<T, I, Epi>, kShortRowsPerBlock, 0));
    per_sm = occ > 0 ? occ : 1;
    constexpr size_t smem = short_pipe_smem_bytes<T, I>();
    MSX_CUDA(cudaFuncSetAttribute(spmv_short_pipe_kernel<T, I, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    occ = 0;
    MSX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmv_short_pipe_kernel<T, I, Epi>,
                                                           kShortRowsPerBlock, smem));
    per_sm_pipe = occ > 0 ? occ : 1;
    sms = num_sms();
    const char *env = getenv("MSX_SPMV_SHORT_PIPE");
    force = env && *env ? atoi(env) : -1;
    cached_dev = dev;
  }
  const int64_t nb = ceil_div(n_rows, kShortRowsPerBlock);
  const int64_t cap = (int64_t)per_sm * sms;
  const bool pipe = force >= 0 ? force != 0 : (Epi::kShortPipe || nb <= kShortPipeMaxBlocks * cap);
  const int64_t cap_used = pipe ? (int64_t)per_sm_pipe * sms : cap;
  return {pipe, nb < cap_used ? nb : cap_used};
}

template <typename T, typename I, typename Epi>
int64_t short_grid(int64_t n_rows) {
  return short_launch<T, I, Epi>(n_rows).grid;
}

inline int64_t binned_blocks(const BinnedPlan &plan) { return plan.info.block_start[kBins]; }

// Persistent grid: at most `waves` full waves of resident CTAs; each CTA walks
// virtual blocks blockIdx.x, +gridDim.x, ...
template <typename T, typename I, typename Epi>
int64_t binned_grid(const BinnedPlan &plan) {
  if (short_rows_plan(plan)) return short_grid<T, I, Epi>(plan.n_rows);
  static thread_local int cached_dev = -1, per_sm = 0, sms = 0;
  int dev = 0;
  MSX_CUDA(cudaGetDevice(&dev));
  if (dev != cached_dev) {
    int occ = 0;
    MSX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmv_binned_kernel<T, I, Epi>, kBinThreads, 0));
    per_sm = occ > 0 ? occ : 1;
    sms = num_sms();
    cached_dev = dev;
  }
  const int64_t cap = (int64_t)per_sm * sms * 4;
  const int64_t nb = binned_blocks(plan);
  return nb < cap ? nb : cap;
}

template <typename T, typename I, typename Epi>
void launch_spmv_binned(const BinnedPlan &plan, const T *data, const I *indices, const I *indptr, const T *x, T *y,
                        float *carry, Epi epi, cudaStream_t stream, bool pdl = false) {
  const int64_t grid = binned_grid<T, I, Epi>(plan);
  if (grid == 0) return;
  if (short_rows_plan(plan)) {
    if (short_launch<T, I, Epi>(plan.n_rows).pipe)
      launch(spmv_short_pipe_kernel<T, I, Epi>, dim3((unsigned)grid), dim3(kShortRowsPerBlock),
             short_pipe_smem_bytes<T, I>(), stream, pdl, data, indices, indptr, x, y, plan.n_rows, plan.nnz, epi);
    else
      launch(spmv_short_kernel<T, I, Epi>, dim3((unsigned)grid), dim3(kShortRowsPerBlock), 0, stream, pdl, data,
             indices, indptr, x, y, plan.n_rows, plan.nnz, epi);
    return;
  }
  launch(spmv_binned_kernel<T, I, Epi>, dim3((unsigned)grid), dim3(kBinThreads), 0, stream, pdl, data, indices, indptr,
         x, y, plan.rows, plan.info, plan.chunk_row, plan.chunk_lo, plan.chunk_hi, carry, epi);
}

template <typename T>
void launch_spmv_long_fixup(const BinnedPlan &plan, const float *carry, T *y, cudaStream_t stream) {
  if (plan.n_long == 0) return;
  spmv_long_fixup_kernel<T><<<(unsigned)ceil_div(plan.n_long, 128), 128, 0, stream>>>(
      plan.rows, plan.info, plan.long_first, carry, y, plan.n_long);
  MSX_CHECK_LAUNCH();
}

// Untyped front door used by the C ABI.
void spmv_binned_run(int value_dtype, int index_dtype, const BinnedPlan &plan, const void *data, const void *indices,
                     const void *indptr, const void *x, void *y, float *carry, cudaStream_t stream);

}  // namespace msx
