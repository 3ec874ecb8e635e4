// SpMV tile machinery shared by the plain product (spmv.cu) and the CG solver
// (cg.cu), which fuses its dot products into the row epilogue.
//
// A "tile" is a contiguous range of the CSR merge path (row ends interleaved
// with nonzeros) of about kTileItems items. Tile boundaries are snapped back to
// row starts unless the row is longer than kSplitRowLen, so short rows are
// always finished inside one tile. See spmv.cu for the algorithm.
//
// Two staging variants feed the same tile walk:
//  - TMA pipeline (default): a persistent CTA keeps two shared-memory stages;
//    while it computes tile j, one elected thread has already issued bulk
//    asynchronous copies (cp.async.bulk, completion on an mbarrier) of tile
//    j+1's column indices, values and row offsets. Requires 16-byte aligned
//    array bases.
//  - direct: coalesced streaming loads into registers, used when a base
//    pointer is not 16-byte aligned.
#pragma once
#include "common.cuh"

namespace msx {

constexpr int kSpmvThreads = 256;
// Path items (rows + nonzeros) per tile before snapping to row starts.
constexpr int kTileItems = 1280;
// Rows longer than this are split between tiles; shorter rows never are.
constexpr int kSplitRowLen = 256;
// Upper bound on a tile's path length after snapping (and so on its nonzeros
// and on its rows).
constexpr int kMaxTileItems = kTileItems + kSplitRowLen;
constexpr int kPerThread = kMaxTileItems / kSpmvThreads;
static_assert(kMaxTileItems % kSpmvThreads == 0, "tile staging assumes whole rounds");

// Bound on mbarrier polling (a safety net; a bulk copy of valid memory
// completes in microseconds).
constexpr long long kMaxPolls = 1ll << 22;

// Merge-path search: number of row ends consumed among the first `diag` path
// items, where row i ends after nonzero row_end(i)-1 (Merrill & Garland).
template <typename Load>
__device__ __forceinline__ int64_t merge_path_search(int64_t diag, int64_t n_a, int64_t n_b, Load row_end) {
  int64_t lo = diag - n_b > 0 ? diag - n_b : 0;
  int64_t hi = diag < n_a ? diag : n_a;
  while (lo < hi) {
    int64_t mid = (lo + hi) >> 1;
    if (row_end(mid) <= diag - mid - 1) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// Rows longer than this inside a tile are summed by a warp; shorter rows by one
// thread, sequentially, in the reference's order.
constexpr int kThreadRowLen = 32;

struct TileSmem {
  float prod[kMaxTileItems];
  int row_end[kMaxTileItems];
  int long_rows[kMaxTileItems / (kThreadRowLen + 1) + 2];
  int n_long;
};

struct TileBounds {
  int64_t r0, r1, k0, k1;
  int R, K;
};

__device__ __forceinline__ TileBounds tile_bounds(int64_t t, const int64_t *tile_row, const int64_t *tile_nz) {
  TileBounds b;
  b.r0 = __ldg(tile_row + t);
  b.r1 = __ldg(tile_row + t + 1);
  b.k0 = __ldg(tile_nz + t);
  b.k1 = __ldg(tile_nz + t + 1);
  b.R = (int)(b.r1 - b.r0);
  b.K = (int)(b.k1 - b.k0);
  return b;
}

// Sums the rows of the staged tile (sm.prod[0..K), sm.row_end[0..R)): a thread
// per row for rows of at most kThreadRowLen nonzeros (summed left to right),
// a warp per longer row (lane-strided, shuffle-tree combine). Row i of the
// tile spans prod[row_end[i-1] .. row_end[i]) (row 0 from 0); a tile that ends
// inside a split row holds that row's head segment as pseudo-row R.
template <typename T, typename I, typename Epi>
__device__ __forceinline__ void tile_rows(int64_t t, const TileBounds &tb, const I *__restrict__ indptr,
                                          T *__restrict__ y, float *__restrict__ carry_head,
                                          float *__restrict__ carry_tail, TileSmem &sm, Epi &epi) {
  const int R = tb.R, K = tb.K;
  const int tid = threadIdx.x;
  const bool head_partial = (R > 0) && (tb.k0 > (int64_t)__ldg(indptr + tb.r0));
  const bool tail_partial = tb.k1 > (int64_t)__ldg(indptr + tb.r1);
  const int n_items = R + (tail_partial ? 1 : 0);
  if (tid == 0) sm.n_long = 0;
  __syncthreads();
  auto emit = [&](int i, float acc) {
    if (i == R) {
      carry_tail[t] = acc;
    } else if (i == 0 && head_partial) {
      carry_head[t] = acc;
    } else {
      const T out = VT<T>::store(acc);
      y[tb.r0 + i] = out;
      epi.row(tb.r0 + i, VT<T>::load(out));
    }
  };
  for (int i = tid; i < n_items; i += kSpmvThreads) {
    const int s = i == 0 ? 0 : sm.row_end[i - 1];
    const int e = i == R ? K : sm.row_end[i];
    if (e - s <= kThreadRowLen) {
      float acc = 0.f;
      for (int j = s; j < e; ++j) acc = add_rn(acc, sm.prod[j]);
      emit(i, acc);
    } else {
      sm.long_rows[atomicAdd(&sm.n_long, 1)] = i;
    }
  }
  __syncthreads();
  const int lane = tid & 31, warp = tid >> 5;
  for (int w = warp; w < sm.n_long; w += kSpmvThreads / 32) {
    const int i = sm.long_rows[w];
    const int s = i == 0 ? 0 : sm.row_end[i - 1];
    const int e = i == R ? K : sm.row_end[i];
    float acc = 0.f;
    for (int j = s + lane; j < e; j += 32) acc = add_rn(acc, sm.prod[j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc = add_rn(acc, __shfl_xor_sync(0xffffffffu, acc, off));
    if (lane == 0) emit(i, acc);
  }
}

// ---- direct staging ----------------------------------------------------------
// Each thread loads its (index, value) pairs of a tile into registers; the
// kernel issues the next tile's loads right after the current tile's products
// are formed, so they are in flight while the rows are summed (2^22-row
// power-law matrix: 0.551 -> 0.533 ms).
template <typename T, typename I>
__device__ __forceinline__ void load_tile_pairs(const TileBounds &tb, const T *__restrict__ data,
                                                const I *__restrict__ indices, I (&col)[kPerThread],
                                                T (&val)[kPerThread]) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int s = 0; s < kPerThread; ++s) {
    const int k = tid + s * kSpmvThreads;
    if (k < tb.K) {
      col[s] = ld_stream(indices + tb.k0 + k);
      val[s] = ld_stream(data + tb.k0 + k);
    }
  }
}

template <typename T, typename I, typename Epi>
__global__ void __launch_bounds__(kSpmvThreads)
spmv_tiles_kernel(const T *__restrict__ data, const I *__restrict__ indices, const I *__restrict__ indptr,
                  const T *__restrict__ x, T *__restrict__ y, const int64_t *__restrict__ tile_row,
                  const int64_t *__restrict__ tile_nz, float *__restrict__ carry_head, float *__restrict__ carry_tail,
                  int64_t n_tiles, Epi epi) {
  __shared__ TileSmem sm;
  if (epi.skip()) return;
  const int tid = threadIdx.x;
  int64_t t = blockIdx.x;
  I col[kPerThread];
  T val[kPerThread];
  TileBounds tb{};
  if (t < n_tiles) {
    tb = tile_bounds(t, tile_row, tile_nz);
    load_tile_pairs<T, I>(tb, data, indices, col, val);
  }
  for (; t < n_tiles; t += gridDim.x) {
#pragma unroll
    for (int s = 0; s < kPerThread; ++s) {
      const int k = tid + s * kSpmvThreads;
      if (k < tb.K) sm.prod[k] = mul_rn(VT<T>::load(val[s]), VT<T>::load(__ldg(x + col[s])));
    }
#pragma unroll
    for (int s = 0; s < kPerThread; ++s) {
      const int i = tid + s * kSpmvThreads;
      if (i < tb.R) sm.row_end[i] = (int)((int64_t)__ldg(indptr + tb.r0 + i + 1) - tb.k0);
    }
    __syncthreads();
    const int64_t t_next = t + gridDim.x;
    TileBounds tb_next{};
    if (t_next < n_tiles) {
      tb_next = tile_bounds(t_next, tile_row, tile_nz);
      load_tile_pairs<T, I>(tb_next, data, indices, col, val);
    }
    tile_rows<T, I, Epi>(t, tb, indptr, y, carry_head, carry_tail, sm, epi);
    __syncthreads();  // smem reused by the next tile
    tb = tb_next;
  }
  epi.finish();
}

// ---- TMA bulk-copy pipeline ------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Global -> shared bulk copy (no multicast); completion counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Waits (at most kMaxPolls polls) for phase `parity` of `bar` to complete, so
// no bulk copy is still writing into shared memory when the CTA exits.
__device__ __forceinline__ void mbar_drain(uint64_t *bar, uint32_t parity) {
  for (long long polls = 0; polls < kMaxPolls && !mbar_try_wait(bar, parity); ++polls) {
  }
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// A 16-byte aligned byte window [lo, hi) of an array that covers elements
// [e0, e1) as far as the array's end allows; elements past `covered` are read
// from global memory instead.
struct BulkWindow {
  uint64_t lo;      // byte offset (from the array base) of the first copied byte
  uint32_t bytes;   // multiple of 16
  uint32_t skew;    // byte offset of element e0 inside the window
  int64_t covered;  // first element index not in the window
};

__device__ __forceinline__ BulkWindow bulk_window(int64_t e0, int64_t e1, int elem, int64_t total_elems) {
  BulkWindow w;
  const uint64_t b0 = (uint64_t)e0 * elem, b1 = (uint64_t)e1 * elem;
  const uint64_t total = (uint64_t)total_elems * elem;
  w.lo = b0 & ~uint64_t(15);
  uint64_t hi = (b1 + 15) & ~uint64_t(15);
  if (hi > total) hi = total & ~uint64_t(15);
  if (hi < w.lo) hi = w.lo;
  w.bytes = (uint32_t)(hi - w.lo);
  w.skew = (uint32_t)(b0 - w.lo);
  const int64_t cov = (int64_t)(hi / elem);
  w.covered = cov < e1 ? cov : e1;
  if (w.covered < e0) w.covered = e0;
  return w;
}

template <typename T, typename I>
struct TmaStage {
  // slack of 16 bytes for the alignment skew of the window start
  alignas(16) unsigned char idx[kMaxTileItems * sizeof(I) + 32];
  alignas(16) unsigned char val[kMaxTileItems * sizeof(T) + 32];
  alignas(16) unsigned char ptr[kMaxTileItems * sizeof(I) + 32];
};

template <typename T, typename I>
struct TmaSmem {
  TmaStage<T, I> stage[2];
  TileSmem tile;
  alignas(8) uint64_t bar[2];
};

template <typename T, typename I>
__device__ __forceinline__ void tma_issue(int64_t t, TmaStage<T, I> &st, uint64_t *bar, const T *data,
                                          const I *indices, const I *indptr, int64_t nnz, int64_t n_rows,
                                          const int64_t *tile_row, const int64_t *tile_nz) {
  const TileBounds tb = tile_bounds(t, tile_row, tile_nz);
  const BulkWindow wi = bulk_window(tb.k0, tb.k1, sizeof(I), nnz);
  const BulkWindow wv = bulk_window(tb.k0, tb.k1, sizeof(T), nnz);
  const BulkWindow wp = bulk_window(tb.r0 + 1, tb.r1 + 1, sizeof(I), n_rows + 1);
  const uint32_t total = wi.bytes + wv.bytes + wp.bytes;
  mbar_arrive_expect_tx(bar, total);
  const char *bi = reinterpret_cast<const char *>(indices);
  const char *bv = reinterpret_cast<const char *>(data);
  const char *bp = reinterpret_cast<const char *>(indptr);
  if (wi.bytes) bulk_g2s(st.idx, bi + wi.lo, wi.bytes, bar);
  if (wv.bytes) bulk_g2s(st.val, bv + wv.lo, wv.bytes, bar);
  if (wp.bytes) bulk_g2s(st.ptr, bp + wp.lo, wp.bytes, bar);
}

// Persistent CTA over tiles blockIdx.x, +gridDim.x, ... with a two-stage TMA
// pipeline. `err` receives 1 if an mbarrier wait exceeds `poll_limit` polls;
// the CTA then stops and the rows of its remaining tiles are not written.
template <typename T, typename I, typename Epi>
__global__ void __launch_bounds__(kSpmvThreads)
spmv_tiles_tma_kernel(const T *__restrict__ data, const I *__restrict__ indices, const I *__restrict__ indptr,
                      const T *__restrict__ x, T *__restrict__ y, const int64_t *__restrict__ tile_row,
                      const int64_t *__restrict__ tile_nz, float *__restrict__ carry_head,
                      float *__restrict__ carry_tail, int64_t n_tiles, int64_t nnz, int64_t n_rows, Epi epi,
                      int *__restrict__ err, long long poll_limit) {
  extern __shared__ __align__(128) unsigned char dyn_smem[];
  TmaSmem<T, I> &sm = *reinterpret_cast<TmaSmem<T, I> *>(dyn_smem);
  const int tid = threadIdx.x;
  int64_t t = blockIdx.x;
  if (t >= n_tiles || epi.skip()) return;
  if (tid == 0) {
    mbar_init(&sm.bar[0], 1);
    mbar_init(&sm.bar[1], 1);
    fence_mbar_init();
    fence_proxy_async_smem();
    tma_issue<T, I>(t, sm.stage[0], &sm.bar[0], data, indices, indptr, nnz, n_rows, tile_row, tile_nz);
  }
  __syncthreads();
  uint32_t phase[2] = {0u, 0u};
  for (int j = 0; t < n_tiles; ++j, t += gridDim.x) {
    const int s = j & 1;
    const int64_t t_next = t + gridDim.x;
    if (tid == 0 && t_next < n_tiles) {
      fence_proxy_async_smem();  // generic reads of the other stage precede its refill
      tma_issue<T, I>(t_next, sm.stage[s ^ 1], &sm.bar[s ^ 1], data, indices, indptr, nnz, n_rows, tile_row,
                      tile_nz);
    }
    // Bounded wait (poll_limit polls; 0 fails at once, which tests use to
    // reach this path). The CTA leaves together: one thread records the
    // timeout and waits, with the fixed bound, for the copies still in flight
    // into this CTA's shared memory before the CTA exits.
    bool done = false;
    for (long long polls = 0; polls < poll_limit && !(done = mbar_try_wait(&sm.bar[s], phase[s])); ++polls) {
    }
    if (__syncthreads_or(!done)) {
      if (tid == 0) {
        atomicOr(err, 1);
        mbar_drain(&sm.bar[s], phase[s]);
        if (t_next < n_tiles) mbar_drain(&sm.bar[s ^ 1], phase[s ^ 1]);
      }
      return;
    }
    phase[s] ^= 1u;

    const TileBounds tb = tile_bounds(t, tile_row, tile_nz);
    const BulkWindow wi = bulk_window(tb.k0, tb.k1, sizeof(I), nnz);
    const BulkWindow wv = bulk_window(tb.k0, tb.k1, sizeof(T), nnz);
    const BulkWindow wp = bulk_window(tb.r0 + 1, tb.r1 + 1, sizeof(I), n_rows + 1);
    const I *sidx = reinterpret_cast<const I *>(sm.stage[s].idx + wi.skew);
    const T *sval = reinterpret_cast<const T *>(sm.stage[s].val + wv.skew);
    const I *sptr = reinterpret_cast<const I *>(sm.stage[s].ptr + wp.skew);
    const int cov_i = (int)(wi.covered - tb.k0), cov_v = (int)(wv.covered - tb.k0);
    const int cov_p = (int)(wp.covered - (tb.r0 + 1));
    {
      I col[kPerThread];
      T val[kPerThread];
#pragma unroll
      for (int q = 0; q < kPerThread; ++q) {
        const int k = tid + q * kSpmvThreads;
        if (k < tb.K) {
          col[q] = k < cov_i ? sidx[k] : indices[tb.k0 + k];
          val[q] = k < cov_v ? sval[k] : data[tb.k0 + k];
        }
      }
#pragma unroll
      for (int q = 0; q < kPerThread; ++q) {
        const int k = tid + q * kSpmvThreads;
        if (k < tb.K) sm.tile.prod[k] = mul_rn(VT<T>::load(val[q]), VT<T>::load(__ldg(x + col[q])));
      }
#pragma unroll
      for (int q = 0; q < kPerThread; ++q) {
        const int i = tid + q * kSpmvThreads;
        if (i < tb.R) {
          const int64_t e = i < cov_p ? (int64_t)sptr[i] : (int64_t)indptr[tb.r0 + 1 + i];
          sm.tile.row_end[i] = (int)(e - tb.k0);
        }
      }
    }
    __syncthreads();
    tile_rows<T, I, Epi>(t, tb, indptr, y, carry_head, carry_tail, sm.tile, epi);
    __syncthreads();  // stage s and the tile arrays are free again
  }
  epi.finish();
}

template <typename T, typename I>
constexpr size_t tma_smem_bytes() {
  return sizeof(TmaSmem<T, I>);
}

int64_t spmv_num_tiles(int64_t n_rows, int64_t nnz);
size_t spmv_plan_device_bytes(int64_t n_tiles);
void spmv_plan_layout(void *base, int64_t n_tiles, int64_t **tile_row, int64_t **tile_nz,
                      unsigned long long **n_split);
void spmv_build_plan(int index_dtype, const void *indptr, int64_t n_rows, int64_t nnz, void *plan_dev,
                     int64_t n_tiles, cudaStream_t stream);
// True when the TMA pipeline can be used for these base pointers.
bool spmv_tma_ok(const void *data, const void *indices, const void *indptr);
// Persistent grid size for the tile kernels on the current device.
template <typename T, typename I, typename Epi>
int spmv_grid_for(int64_t n_tiles, bool tma);
int spmv_grid(int64_t n_tiles);
// Device int the TMA kernels flag when an mbarrier wait times out (per device;
// sticky until msx_check_device_errors reads and clears it).
int *spmv_error_flag();
// Poll bound of the TMA kernels' mbarrier waits (kMaxPolls unless changed by
// msx_debug_set_spmv_poll_limit).
long long spmv_poll_limit();
// Sets it (a negative value restores kMaxPolls); process-wide.
void spmv_set_poll_limit(long long polls);
// Reads and clears the current device's timeout flag.
bool spmv_take_error();
// carry_scratch: float[2*n_tiles] when launch_fixup, else may be null.
void spmv_run(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
              const void *x, void *y, int64_t n_rows, int64_t nnz, const void *plan_dev, int64_t n_tiles,
              bool launch_fixup, float *carry_scratch, cudaStream_t stream);
// Fixup of split rows for fp32 y (used by the solvers).
void spmv_fixup_f32(int index_dtype, const void *indptr, float *y, const void *plan_dev, int64_t n_tiles,
                    const float *carry_scratch, cudaStream_t stream);

// Launches the tile kernel (TMA pipeline when the pointers allow) with an
// epilogue; shared by spmv.cu and cg.cu.
template <typename T, typename I, typename Epi>
void launch_spmv_tiles(const T *data, const I *indices, const I *indptr, const T *x, T *y, const int64_t *tile_row,
                       const int64_t *tile_nz, float *carry_head, float *carry_tail, int64_t n_tiles, int64_t nnz,
                       int64_t n_rows, Epi epi, cudaStream_t stream) {
  if (n_tiles == 0) return;
  const bool tma = spmv_tma_ok(data, indices, indptr);
  const int grid = spmv_grid_for<T, I, Epi>(n_tiles, tma);
  if (tma) {
    spmv_tiles_tma_kernel<T, I, Epi><<<grid, kSpmvThreads, tma_smem_bytes<T, I>(), stream>>>(
        data, indices, indptr, x, y, tile_row, tile_nz, carry_head, carry_tail, n_tiles, nnz, n_rows, epi,
        spmv_error_flag(), spmv_poll_limit());
  } else {
    spmv_tiles_kernel<T, I, Epi><<<grid, kSpmvThreads, 0, stream>>>(data, indices, indptr, x, y, tile_row, tile_nz,
                                                                    carry_head, carry_tail, n_tiles, epi);
  }
  MSX_CHECK_LAUNCH();
}

template <typename T, typename I, typename Epi>
int spmv_grid_for(int64_t n_tiles, bool tma) {
  static thread_local int cached_dev[2] = {-1, -1}, per_sm[2] = {0, 0}, sms = 0;
  int dev = 0;
  MSX_CUDA(cudaGetDevice(&dev));
  const int v = tma ? 1 : 0;
  if (dev != cached_dev[v]) {
    int occ = 0;
    if (tma) {
      auto kern = spmv_tiles_tma_kernel<T, I, Epi>;
      MSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tma_smem_bytes<T, I>()));
      MSX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kSpmvThreads, tma_smem_bytes<T, I>()));
    } else {
      MSX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, spmv_tiles_kernel<T, I, Epi>, kSpmvThreads, 0));
    }
    per_sm[v] = occ > 0 ? occ : 1;
    sms = num_sms();
    cached_dev[v] = dev;
  }
  const int64_t g = (int64_t)per_sm[v] * sms;
  return (int)(n_tiles < g ? n_tiles : g);
}

}  // namespace msx
