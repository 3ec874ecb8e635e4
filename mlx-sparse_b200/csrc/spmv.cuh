// SpMV tile machinery shared by the plain product (spmv.cu) and the CG solver
// (cg.cu), which fuses its dot products into the row epilogue.
//
// A "tile" is a contiguous range of the CSR merge path (row ends interleaved
// with nonzeros) of about kTileItems items. Tile boundaries are snapped back to
// row starts unless the row is longer than kSplitRowLen, so short rows are
// always finished inside one tile. See spmv.cu for the algorithm.
#pragma once
#include "common.cuh"

namespace msx {

constexpr int kSpmvThreads = 256;
// Path items (rows + nonzeros) per tile before snapping to row starts.
constexpr int kTileItems = 1536;
// Rows longer than this are split between tiles; shorter rows never are.
constexpr int kSplitRowLen = kTileItems / 2;
// Upper bound on a tile's path length after snapping.
constexpr int kMaxTileItems = kTileItems + kSplitRowLen;
static_assert(kMaxTileItems % kSpmvThreads == 0, "tile staging assumes whole rounds");

struct SegPair {
  int flag;  // 1 if the segment contains a row end (resets the running sum)
  float val;
};

__device__ __forceinline__ SegPair seg_combine(SegPair a, SegPair b) {
  // a precedes b
  SegPair r;
  r.flag = a.flag | b.flag;
  r.val = b.flag ? b.val : add_rn(a.val, b.val);
  return r;
}

// Block-wide exclusive segmented scan over kSpmvThreads threads.
__device__ __forceinline__ SegPair block_exclusive_seg_scan(SegPair v, SegPair *warp_tot) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  constexpr int kWarps = kSpmvThreads / 32;
  SegPair inc = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    SegPair o;
    o.flag = __shfl_up_sync(0xffffffffu, inc.flag, off);
    o.val = __shfl_up_sync(0xffffffffu, inc.val, off);
    if (lane >= off) inc = seg_combine(o, inc);
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    SegPair w = lane < kWarps ? warp_tot[lane] : SegPair{0, 0.f};
#pragma unroll
    for (int off = 1; off < kWarps; off <<= 1) {
      SegPair o;
      o.flag = __shfl_up_sync(0xffffffffu, w.flag, off);
      o.val = __shfl_up_sync(0xffffffffu, w.val, off);
      if (lane >= off) w = seg_combine(o, w);
    }
    if (lane < kWarps) warp_tot[lane] = w;  // inclusive prefixes over warps
  }
  __syncthreads();
  SegPair prev_lanes;
  prev_lanes.flag = __shfl_up_sync(0xffffffffu, inc.flag, 1);
  prev_lanes.val = __shfl_up_sync(0xffffffffu, inc.val, 1);
  SegPair ex;
  if (lane == 0) {
    ex = warp > 0 ? warp_tot[warp - 1] : SegPair{0, 0.f};
  } else {
    ex = warp > 0 ? seg_combine(warp_tot[warp - 1], prev_lanes) : prev_lanes;
  }
  __syncthreads();  // warp_tot is reused by the next tile
  return ex;
}

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

struct TileSmem {
  float prod[kMaxTileItems];
  int row_end[kMaxTileItems];
  SegPair warp_tot[kSpmvThreads / 32];
};

// Epilogue that only stores y.
struct NoEpilogue {
  __device__ __forceinline__ void row(int64_t, float) {}
};

// Processes tile t: y[r] for every row finished in the tile, tile partials of
// split rows into carry_head / carry_tail. Must be called by all kSpmvThreads.
template <typename T, typename I, typename Epi>
__device__ __forceinline__ void spmv_process_tile(int64_t t, const T *__restrict__ data, const I *__restrict__ indices,
                                                  const I *__restrict__ indptr, const T *__restrict__ x,
                                                  T *__restrict__ y, const int64_t *__restrict__ tile_row,
                                                  const int64_t *__restrict__ tile_nz, float *__restrict__ carry_head,
                                                  float *__restrict__ carry_tail, TileSmem &sm, Epi &epi) {
  const int64_t r0 = tile_row[t], r1 = tile_row[t + 1];
  const int64_t k0 = tile_nz[t], k1 = tile_nz[t + 1];
  const int R = (int)(r1 - r0);  // rows whose end lies in this tile
  const int K = (int)(k1 - k0);  // nonzeros in this tile
  const int P = R + K;
  const int tid = threadIdx.x;
  const int64_t head_start = (int64_t)__ldg(indptr + r0);
  const int64_t tail_start = (int64_t)__ldg(indptr + r1);

  // Stage products and row ends: every load of the tile is issued before any
  // is consumed.
  {
    constexpr int kPer = kMaxTileItems / kSpmvThreads;
    I col[kPer];
    T val[kPer];
#pragma unroll
    for (int s = 0; s < kPer; ++s) {
      const int k = tid + s * kSpmvThreads;
      if (k < K) {
        col[s] = ld_stream(indices + k0 + k);
        val[s] = ld_stream(data + k0 + k);
      }
    }
#pragma unroll
    for (int s = 0; s < kPer; ++s) {
      const int k = tid + s * kSpmvThreads;
      if (k < K) sm.prod[k] = mul_rn(VT<T>::load(val[s]), VT<T>::load(__ldg(x + col[s])));
    }
#pragma unroll
    for (int s = 0; s < kPer; ++s) {
      const int i = tid + s * kSpmvThreads;
      if (i < R) sm.row_end[i] = (int)((int64_t)__ldg(indptr + r0 + i + 1) - k0);
    }
  }
  __syncthreads();

  const bool head_partial = (R > 0) && (k0 > head_start);
  const int ipt = (P + kSpmvThreads - 1) / kSpmvThreads;
  const int d0 = min(tid * ipt, P);
  const int d1 = min(d0 + ipt, P);
  const int i0 = (int)merge_path_search(d0, R, K, [&](int64_t i) { return (int64_t)sm.row_end[i]; });
  const int j0 = d0 - i0;

  // Pass 1: this thread's carry-out (sum after its last row end).
  SegPair mine{0, 0.f};
  {
    int i = i0, j = j0;
    float acc = 0.f;
    for (int d = d0; d < d1; ++d) {
      if (i < R && sm.row_end[i] <= j) {
        mine.flag = 1;
        acc = 0.f;
        ++i;
      } else {
        acc = add_rn(acc, sm.prod[j]);
        ++j;
      }
    }
    mine.val = acc;
  }
  const SegPair carry = block_exclusive_seg_scan(mine, sm.warp_tot);

  // Pass 2: re-walk from the carried-in partial and write the rows.
  {
    int i = i0, j = j0;
    float acc = carry.val;
    for (int d = d0; d < d1; ++d) {
      if (i < R && sm.row_end[i] <= j) {
        if (i == 0 && head_partial) {
          carry_head[t] = acc;
        } else {
          const T out = VT<T>::store(acc);
          y[r0 + i] = out;
          epi.row(r0 + i, VT<T>::load(out));
        }
        acc = 0.f;
        ++i;
      } else {
        acc = add_rn(acc, sm.prod[j]);
        ++j;
      }
    }
    // The thread holding the last path item owns the tile's tail partial when
    // the tile ends inside a (split) row.
    if (d0 < d1 && d1 == P && k1 > tail_start) carry_tail[t] = acc;
  }
  __syncthreads();  // smem reused by the next tile
}

template <typename T, typename I, typename Epi>
__global__ void __launch_bounds__(kSpmvThreads)
spmv_tiles_kernel(const T *__restrict__ data, const I *__restrict__ indices, const I *__restrict__ indptr,
                  const T *__restrict__ x, T *__restrict__ y, const int64_t *__restrict__ tile_row,
                  const int64_t *__restrict__ tile_nz, float *__restrict__ carry_head, float *__restrict__ carry_tail,
                  int64_t n_tiles, Epi epi) {
  __shared__ TileSmem sm;
  for (int64_t t = blockIdx.x; t < n_tiles; t += gridDim.x) {
    spmv_process_tile<T, I, Epi>(t, data, indices, indptr, x, y, tile_row, tile_nz, carry_head, carry_tail, sm, epi);
  }
}

int64_t spmv_num_tiles(int64_t n_rows, int64_t nnz);
size_t spmv_plan_device_bytes(int64_t n_tiles);
void spmv_plan_layout(void *base, int64_t n_tiles, int64_t **tile_row, int64_t **tile_nz,
                      unsigned long long **n_split);
void spmv_build_plan(int index_dtype, const void *indptr, int64_t n_rows, int64_t nnz, void *plan_dev,
                     int64_t n_tiles, cudaStream_t stream);
// Persistent grid size for the tile kernel on the current device.
int spmv_grid(int64_t n_tiles);
// carry_scratch: float[2*n_tiles] when launch_fixup, else may be null.
void spmv_run(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
              const void *x, void *y, int64_t n_rows, const void *plan_dev, int64_t n_tiles, bool launch_fixup,
              float *carry_scratch, cudaStream_t stream);
// Fixup of split rows for fp32 y (used by the solvers).
void spmv_fixup_f32(int index_dtype, const void *indptr, float *y, const void *plan_dev, int64_t n_tiles,
                    const float *carry_scratch, cudaStream_t stream);

}  // namespace msx
