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
// B200 design: one expansion pass over rows binned by their product count W,
// writing every finished row (sorted, summed, pruned) into a temporary buffer
// at an upper-bound offset (the prefix sum of W), then a scan of the exact row
// counts gives indptr; the numeric call of the two-call protocol only copies
// the rows into the caller's arrays. Rows are processed by
//   W <= 256     one warp: the row's lhs entries and their rhs row bounds are
//                read by the lanes in parallel (one round trip), each lane
//                expands its products with a shuffle search over the prefix of
//                rhs row lengths, so every gather of the row is in flight at
//                once; the 64-bit keys (column << 32 | position) are
//                bitonic-sorted in shared memory and each column's run is
//                summed in position order - the reference's exact
//                accumulation order - and compacted with warp ballots;
//   W <= 4096    the same with one CTA per row;
//   W  > 4096    one CTA per row over a dense global accumulator (marker +
//                value per column): lhs entries are applied one after another,
//                the entries of one rhs row in parallel (rhs rows without
//                repeated columns) or by one thread (otherwise), then columns
//                are extracted in ascending order.
// The symbolic call synchronises twice (the total product count sizes the
// temporary buffer; the output nnz is returned) and keeps the finished rows
// for the numeric call on the same thread, which then needs no recomputation
// (it recomputes only if the cached product does not match its arguments).
// No atomics touch values, so results are deterministic.
#include <algorithm>
#include <memory>
#include <type_traits>
#include <vector>

#include "common.cuh"
#include "scan.cuh"

namespace msx {

namespace {

constexpr int kWarpCap = 256;    // products per warp-level row
constexpr int kBlockCap = 4096;  // products per CTA-level row
constexpr int kBlockThreads = 256;
constexpr int kDenseThreads = 512;
constexpr int kBins = 8;  // smem warp, CTA, dense, register warp R = 1, 2, 4, 8, four rows per warp

__device__ __forceinline__ uint32_t key_col(uint64_t k) { return (uint32_t)(k >> 32); }
__device__ __forceinline__ uint32_t key_seq(uint64_t k) { return (uint32_t)(k & 0xffffffffu); }

// ---- row work, checks and binning --------------------------------------------
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

// Appends every row to the list of its bin. The lanes of a warp that fall in
// the same bin take their slots with one atomic per bin and warp (a single
// counter hit by every row serialises).
template <typename LI>
__global__ void bin_kernel(const int64_t *__restrict__ work, const LI *__restrict__ lp, int64_t m, bool reg_ok,
                           bool quad_ok, int *__restrict__ lists, int *__restrict__ counts,
                           int64_t *__restrict__ row_nnz) {
  const int64_t row = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int lane = threadIdx.x & 31;
  int bin = -1;
  if (row < m) {
    const int64_t w = work[row];
    if (w == 0) {
      row_nnz[row] = 0;
    } else if (w <= kWarpCap) {
      // bin 7: four rows per warp (<= 64 products, <= 8 lhs entries each);
      // bins 3..6: one warp with the keys in 1, 2, 4 or 8 registers per lane
      // (<= 32 lhs entries); else the shared-memory warp path
      const int64_t nq = (int64_t)lp[row + 1] - (int64_t)lp[row];
      if (quad_ok && w <= 64 && nq <= 8)
        bin = 7;
      else if (reg_ok && nq <= 32)
        bin = w <= 32 ? 3 : (w <= 64 ? 4 : (w <= 128 ? 5 : 6));
      else
        bin = 0;
    } else {
      bin = w <= kBlockCap ? 1 : 2;
    }
  }
#pragma unroll
  for (int b = 0; b < kBins; ++b) {
    const unsigned mask = __ballot_sync(0xffffffffu, bin == b);
    if (mask == 0) continue;
    const int leader = __ffs(mask) - 1;
    int base = 0;
    if (lane == leader) base = atomicAdd(counts + b, __popc(mask));
    base = __shfl_sync(0xffffffffu, base, leader);
    if (bin == b) lists[b * m + base + __popc(mask & ((1u << lane) - 1u))] = (int)row;
  }
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

// Where finished rows go: at the row's upper-bound offset in the temporary
// arrays (column as int32, value as T); row_nnz receives the exact count.
template <typename T>
struct RowSink {
  const int64_t *off;
  int *col;
  T *val;
  int64_t *row_nnz;
};

// Sorts the cnt keys (already in shared memory), sums every column's run in
// position order, prunes exact zeros and writes the row to the sink.
template <typename T, bool kWarp>
__device__ void compact_sorted_row(int64_t row, int cnt, int tid, int nthreads, const uint64_t *key,
                                   const float *val, int *scratch_cnt, RowSink<T> sink, bool prune);

template <typename T, bool kWarp>
__device__ void finish_row(int64_t row, int cnt, int tid, int nthreads, uint64_t *key, const float *val,
                           int *scratch_cnt, RowSink<T> sink, bool prune) {
  auto sync = [&]() {
    if (kWarp) __syncwarp();
    else __syncthreads();
  };
  int pw = 1;
  while (pw < cnt) pw <<= 1;
  for (int j = cnt + tid; j < pw; j += nthreads) key[j] = ~0ull;
  sync();
  bitonic_sort(key, pw, tid, nthreads, sync);
  compact_sorted_row<T, kWarp>(row, cnt, tid, nthreads, key, val, scratch_cnt, sink, prune);
}

// Sums each column's run of the sorted keys in position order, prunes exact
// zeros and writes the row to the sink.
template <typename T, bool kWarp>
__device__ void compact_sorted_row(int64_t row, int cnt, int tid, int nthreads, const uint64_t *key,
                                   const float *val, int *scratch_cnt, RowSink<T> sink, bool prune) {
  auto sync = [&]() {
    if (kWarp) __syncwarp();
    else __syncthreads();
  };
  const int64_t out0 = sink.off[row];
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
    if (keep) {
      sink.col[out0 + pos] = (int)col;
      sink.val[out0 + pos] = out_v;
    }
  }
  if (tid == 0) sink.row_nnz[row] = count;
  sync();
}

// One warp per row with W <= kWarpCap products. The lanes read up to 32 lhs
// entries of the row and their rhs row bounds at once; a warp-wide prefix sum
// of the rhs row lengths lets every lane find, by a shuffle search, which lhs
// entry each of its products belongs to, so all the row's rhs gathers are in
// flight together. Rows with more than 32 lhs entries take the entries in
// chunks of 32.
template <typename T, typename LI, typename RI>
__global__ void __launch_bounds__(kBlockThreads)
spgemm_warp_kernel(const int *__restrict__ list, const int *__restrict__ count_ptr, const int *__restrict__ flags,
                   const T *__restrict__ ld, const LI *__restrict__ li, const LI *__restrict__ lp,
                   const T *__restrict__ rd, const RI *__restrict__ ri, const RI *__restrict__ rp, RowSink<T> sink,
                   bool prune) {
  __shared__ uint64_t keys[kBlockThreads / 32][kWarpCap];
  __shared__ float vals[kBlockThreads / 32][kWarpCap];
  if (*flags & 3) return;  // invalid indices: the host reports them
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int count = *count_ptr;
  uint64_t *key = keys[warp];
  float *val = vals[warp];
  for (int w = blockIdx.x * (kBlockThreads / 32) + warp; w < count; w += gridDim.x * (kBlockThreads / 32)) {
    const int64_t row = list[w];
    const int64_t q0 = (int64_t)lp[row], q1 = (int64_t)lp[row + 1];
    int cnt = 0;
    for (int64_t qc = q0; qc < q1; qc += 32) {
      const int nq = (int)min((int64_t)32, q1 - qc);
      int64_t rb = 0;
      int len = 0;
      float lv = 0.f;
      if (lane < nq) {
        const int64_t k = (int64_t)li[qc + lane];
        lv = VT<T>::load(ld[qc + lane]);
        rb = (int64_t)rp[k];
        len = (int)((int64_t)rp[k + 1] - rb);
      }
      int incl = len;  // inclusive prefix of the lengths over the lanes
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      const int chunk = __shfl_sync(0xffffffffu, incl, 31);
      // all lanes run every round (the shuffles need the full warp)
      for (int base = 0; base < chunk; base += 32) {
        const int s = base + lane;
        // e = number of entries whose inclusive prefix is <= s, i.e. the
        // entry product s belongs to (binary lifting over the lanes)
        int e = 0;
#pragma unroll
        for (int b = 16; b > 0; b >>= 1) {
          const int v = __shfl_sync(0xffffffffu, incl, (e + b - 1) & 31);
          if (e + b <= nq && v <= s) e += b;
        }
        const int ev = e & 31;
        const int excl = __shfl_sync(0xffffffffu, incl, ev) - __shfl_sync(0xffffffffu, len, ev);
        const int64_t erb = __shfl_sync(0xffffffffu, rb, ev);
        const float elv = __shfl_sync(0xffffffffu, lv, ev);
        if (s < chunk) {
          const int64_t src = erb + (s - excl);
          const int pos = cnt + s;
          key[pos] = ((uint64_t)(uint32_t)ri[src] << 32) | (uint32_t)pos;
          val[pos] = __fmul_rn(elv, VT<T>::load(rd[src]));
        }
      }
      cnt += chunk;
    }
    __syncwarp();
    finish_row<T, true>(row, cnt, lane, 32, key, val, nullptr, sink, prune);
  }
}

// Rows of W <= 32 R products and at most 32 lhs entries, with the sort keys
// in registers: key = column << 8 | position (n_cols < 2^24, W <= 256), one
// key per lane and register, element i = lane * R + r of a bitonic network
// whose cross-lane stages are shuffles. A row without repeated columns is
// then compacted straight from the registers; a row with repeats takes the
// shared-memory run summation.
template <typename T, int R>
__device__ __forceinline__ void reg_sort_row(int64_t row, int W, uint32_t (&key)[R], uint64_t *skey,
                                             const float *val, RowSink<T> sink, bool prune) {
  const int lane = threadIdx.x & 31;
  constexpr int N = 32 * R;
#pragma unroll
  for (int k = 2; k <= N; k <<= 1) {
#pragma unroll
    for (int j = k >> 1; j > 0; j >>= 1) {
      if (j >= R) {
        const int lm = j / R;
        const bool lower = (lane & lm) == 0;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint32_t other = __shfl_xor_sync(0xffffffffu, key[r], lm);
          const bool up = (((lane * R + r) & k) == 0);
          key[r] = (lower == up) ? min(key[r], other) : max(key[r], other);
        }
      } else {
#pragma unroll
        for (int r = 0; r < R; ++r) {
          if ((r & j) == 0) {
            const bool up = (((lane * R + r) & k) == 0);
            const uint32_t a = key[r], b = key[r | j];
            if ((a > b) == up) {
              key[r] = b;
              key[r | j] = a;
            }
          }
        }
      }
    }
  }
  // repeated columns (rare for random patterns): sum runs in shared memory
  const uint32_t next_first = __shfl_down_sync(0xffffffffu, key[0], 1);
  bool dup = false;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = lane * R + r;
    const uint32_t nk = r + 1 < R ? key[r + 1] : next_first;
    if (i + 1 < W && (key[r] >> 8) == (nk >> 8)) dup = true;
  }
  if (__any_sync(0xffffffffu, dup)) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int i = lane * R + r;
      if (i < W) skey[i] = ((uint64_t)(key[r] >> 8) << 32) | (key[r] & 0xffu);
    }
    __syncwarp();
    compact_sorted_row<T, true>(row, W, lane, 32, skey, val, nullptr, sink, prune);
    return;
  }
  bool keep[R];
  T outv[R];
  int mine = 0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = lane * R + r;
    keep[r] = false;
    if (i < W) {
      outv[r] = VT<T>::store(val[key[r] & 0xffu]);
      keep[r] = !prune || VT<T>::load(outv[r]) != 0.0f;
    }
    mine += keep[r] ? 1 : 0;
  }
  int incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  int64_t pos = sink.off[row] + (incl - mine);
#pragma unroll
  for (int r = 0; r < R; ++r)
    if (keep[r]) {
      sink.col[pos] = (int)(key[r] >> 8);
      sink.val[pos] = outv[r];
      ++pos;
    }
  if (lane == 31) sink.row_nnz[row] = incl;
  __syncwarp();
}

template <typename T, typename LI, typename RI, int R>
__global__ void __launch_bounds__(kBlockThreads)
spgemm_warp_reg_kernel(const int *__restrict__ list, const int *__restrict__ count_ptr, const int *__restrict__ flags,
                       const int64_t *__restrict__ work, const T *__restrict__ ld, const LI *__restrict__ li,
                       const LI *__restrict__ lp, const T *__restrict__ rd, const RI *__restrict__ ri,
                       const RI *__restrict__ rp, RowSink<T> sink, bool prune) {
  __shared__ uint64_t keys[kBlockThreads / 32][kWarpCap];
  __shared__ float vals[kBlockThreads / 32][kWarpCap];
  if (*flags & 3) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int count = *count_ptr;
  float *val = vals[warp];
  for (int w = blockIdx.x * (kBlockThreads / 32) + warp; w < count; w += gridDim.x * (kBlockThreads / 32)) {
    const int64_t row = list[w];
    const int W = (int)work[row];
    const int64_t q0 = (int64_t)lp[row];
    const int nq = (int)((int64_t)lp[row + 1] - q0);
    int64_t rb = 0;
    int len = 0;
    float lv = 0.f;
    if (lane < nq) {
      const int64_t k = (int64_t)li[q0 + lane];
      lv = VT<T>::load(ld[q0 + lane]);
      rb = (int64_t)rp[k];
      len = (int)((int64_t)rp[k + 1] - rb);
    }
    int incl = len;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    // product s = 32 u + lane goes to register u
    uint32_t key[R];
#pragma unroll
    for (int u = 0; u < R; ++u) {
      const int s = 32 * u + lane;
      int e = 0;
#pragma unroll
      for (int b = 16; b > 0; b >>= 1) {
        const int v = __shfl_sync(0xffffffffu, incl, (e + b - 1) & 31);
        if (e + b <= nq && v <= s) e += b;
      }
      const int ev = e & 31;
      const int excl = __shfl_sync(0xffffffffu, incl, ev) - __shfl_sync(0xffffffffu, len, ev);
      const int64_t erb = __shfl_sync(0xffffffffu, rb, ev);
      const float elv = __shfl_sync(0xffffffffu, lv, ev);
      key[u] = ~0u;
      if (s < W) {
        const int64_t src = erb + (s - excl);
        key[u] = ((uint32_t)ri[src] << 8) | (uint32_t)s;
        val[s] = __fmul_rn(elv, VT<T>::load(rd[src]));
      }
    }
    __syncwarp();
    reg_sort_row<T, R>(row, W, key, keys[warp], val, sink, prune);
  }
}

// Four rows per warp, each with <= 64 products and <= 8 lhs entries: row g
// of the four owns lanes 8g..8g+7. Those lanes hold its lhs entries and rhs
// row bounds (one round trip of index loads serves four rows), then its 64
// key slots, 8 registers per lane, with the keys column << 8 | position
// (padding all ones). Lane e of the group expands products e, e + 8, ...,
// so a group's loads of one rhs row are consecutive. A bitonic sort whose
// stages stop at 64 keys orders each group's segment on its own (21 stages,
// 3 of them across lanes). Rows without repeated columns are compacted from
// the registers through a shared-memory staging slot (so the stores of a row
// are consecutive); if any row of the four repeats a column, the four rows
// take the shared-memory run summation one after another.
template <typename T, typename LI, typename RI>
__global__ void __launch_bounds__(kBlockThreads, 4)  // 64 registers: 4 CTAs/SM (80 unbounded: 3; 161 -> 145 us)
spgemm_quad_kernel(const int *__restrict__ list, const int *__restrict__ count_ptr, const int *__restrict__ flags,
                   const int64_t *__restrict__ work, const T *__restrict__ ld, const LI *__restrict__ li,
                   const LI *__restrict__ lp, const T *__restrict__ rd, const RI *__restrict__ ri,
                   const RI *__restrict__ rp, RowSink<T> sink, bool prune) {
  __shared__ uint64_t keys[kBlockThreads / 32][64];
  __shared__ float vals[kBlockThreads / 32][256];
  __shared__ int cols[kBlockThreads / 32][256];
  if (*flags & 3) return;
  constexpr int R = 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g_mine = lane >> 3, e_mine = lane & 7, base = g_mine * 8;
  const int count = *count_ptr;
  const int n_quads = (count + 3) / 4;
  float *val = vals[warp];
  float *my_val = val + g_mine * 64;
  for (int w = blockIdx.x * (kBlockThreads / 32) + warp; w < n_quads; w += gridDim.x * (kBlockThreads / 32)) {
    const int li_idx = 4 * w + g_mine;  // slots past the list's end stay empty
    const int64_t my_row = li_idx < count ? (int64_t)list[li_idx] : -1;
    int rw = 0, nq = 0;
    int64_t q0 = 0;
    if (my_row >= 0) {
      rw = (int)work[my_row];
      q0 = (int64_t)lp[my_row];
      nq = (int)((int64_t)lp[my_row + 1] - q0);
    }
    int64_t rb = 0;
    int len = 0;
    float lv = 0.f;
    if (e_mine < nq) {
      const int64_t k = (int64_t)li[q0 + e_mine];
      lv = VT<T>::load(ld[q0 + e_mine]);
      rb = (int64_t)rp[k];
      len = (int)((int64_t)rp[k + 1] - rb);
    }
    int incl = len;  // inclusive prefix over the group's 8 lanes
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o, 8);
      if (e_mine >= o) incl += v;
    }
    uint32_t key[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int t = r * 8 + e_mine;  // product position within the row
      int e = 0;
#pragma unroll
      for (int b = 4; b > 0; b >>= 1) {
        const int v = __shfl_sync(0xffffffffu, incl, base + ((e + b - 1) & 7));
        if (e + b <= nq && v <= t) e += b;
      }
      const int src_lane = base + (e & 7);
      const int excl = __shfl_sync(0xffffffffu, incl, src_lane) - __shfl_sync(0xffffffffu, len, src_lane);
      const int64_t erb = __shfl_sync(0xffffffffu, rb, src_lane);
      const float elv = __shfl_sync(0xffffffffu, lv, src_lane);
      key[r] = 0xffffffffu;
      if (t < rw) {
        const int64_t src = erb + (t - excl);
        key[r] = ((uint32_t)ri[src] << 8) | (uint32_t)t;
        my_val[t] = __fmul_rn(elv, VT<T>::load(rd[src]));
      }
    }
    __syncwarp();
    // element i = lane * R + r; every stage sorts within aligned 64-key
    // segments, all ascending
#pragma unroll
    for (int k = 2; k <= 64; k <<= 1) {
#pragma unroll
      for (int j = k >> 1; j > 0; j >>= 1) {
        if (j >= R) {
          const int lm = j / R;
          const bool lower = (lane & lm) == 0;
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const uint32_t other = __shfl_xor_sync(0xffffffffu, key[r], lm);
            const bool up = k == 64 || (((lane * R + r) & k) == 0);
            key[r] = (lower == up) ? min(key[r], other) : max(key[r], other);
          }
        } else {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            if ((r & j) == 0) {
              const bool up = k == 64 || (((lane * R + r) & k) == 0);
              const uint32_t a = key[r], b = key[r | j];
              if ((a > b) == up) {
                key[r] = b;
                key[r | j] = a;
              }
            }
          }
        }
      }
    }
    // this lane holds positions e_mine * R .. e_mine * R + 7 of its row
    const uint32_t next_first = __shfl_down_sync(0xffffffffu, key[0], 1);
    bool dup = false;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int i = e_mine * R + r;
      const uint32_t nk = r + 1 < R ? key[r + 1] : next_first;
      if (i + 1 < rw && (key[r] >> 8) == (nk >> 8)) dup = true;
    }
    if (__any_sync(0xffffffffu, dup)) {
      // every row of the quad through the shared-memory run summation
      for (int g = 0; g < 4; ++g) {
        const int64_t row = __shfl_sync(0xffffffffu, my_row, g * 8);
        const int W = __shfl_sync(0xffffffffu, rw, g * 8);
        if (row < 0) continue;
        __syncwarp();  // the previous row's summation has finished reading keys
        if (g_mine == g) {
#pragma unroll
          for (int r = 0; r < R; ++r) {
            const int i = e_mine * R + r;
            if (i < W) keys[warp][i] = ((uint64_t)(key[r] >> 8) << 32) | (key[r] & 0xffu);
          }
        }
        __syncwarp();
        compact_sorted_row<T, true>(row, W, lane, 32, keys[warp], val + g * 64, nullptr, sink, prune);
      }
      __syncwarp();
      continue;
    }
    bool keep[R];
    T outv[R];
    int mine = 0;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int i = e_mine * R + r;
      keep[r] = false;
      if (i < rw) {
        outv[r] = VT<T>::store(my_val[key[r] & 0xffu]);
        keep[r] = !prune || VT<T>::load(outv[r]) != 0.0f;
      }
      mine += keep[r] ? 1 : 0;
    }
    int incl_k = mine;
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl_k, o, 8);
      if (e_mine >= o) incl_k += v;
    }
    // stage the compacted row in shared memory (the values were read into
    // registers above), then the group's 8 lanes write it out consecutively
    __syncwarp();
    T *st_val = reinterpret_cast<T *>(my_val);
    int *st_col = cols[warp] + g_mine * 64;
    int pos = incl_k - mine;
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (keep[r]) {
        st_col[pos] = (int)(key[r] >> 8);
        st_val[pos] = outv[r];
        ++pos;
      }
    __syncwarp();
    const int cnt = __shfl_sync(0xffffffffu, incl_k, base + 7);
    if (my_row >= 0) {
      const int64_t out0 = sink.off[my_row];
      for (int j = e_mine; j < cnt; j += 8) {
        sink.col[out0 + j] = st_col[j];
        sink.val[out0 + j] = st_val[j];
      }
      if (e_mine == 7) sink.row_nnz[my_row] = cnt;
    }
    __syncwarp();
  }
}

template <typename T, typename LI, typename RI>
__global__ void __launch_bounds__(kBlockThreads)
spgemm_block_kernel(const int *__restrict__ list, const int *__restrict__ count_ptr, const int *__restrict__ flags,
                    const T *__restrict__ ld, const LI *__restrict__ li, const LI *__restrict__ lp,
                    const T *__restrict__ rd, const RI *__restrict__ ri, const RI *__restrict__ rp, RowSink<T> sink,
                    bool prune) {
  extern __shared__ __align__(16) unsigned char dyn[];
  uint64_t *key = reinterpret_cast<uint64_t *>(dyn);
  float *val = reinterpret_cast<float *>(key + kBlockCap);
  __shared__ int cnt_s[kBlockThreads / 32];
  if (*flags & 3) return;
  const int count = *count_ptr;
  const int tid = threadIdx.x;
  for (int b = blockIdx.x; b < count; b += gridDim.x) {
    const int64_t row = list[b];
    // expand in (lhs position, rhs position) order
    int cnt = 0;
    for (int64_t q = (int64_t)lp[row]; q < (int64_t)lp[row + 1]; ++q) {
      const int64_t k = (int64_t)li[q];
      const float lv = VT<T>::load(ld[q]);
      const int64_t rb = (int64_t)rp[k];
      const int len = (int)((int64_t)rp[k + 1] - rb);
      for (int j = tid; j < len; j += kBlockThreads) {
        const int s = cnt + j;
        key[s] = ((uint64_t)(uint32_t)ri[rb + j] << 32) | (uint32_t)s;
        val[s] = __fmul_rn(lv, VT<T>::load(rd[rb + j]));
      }
      cnt += len;
    }
    __syncthreads();
    finish_row<T, false>(row, cnt, tid, kBlockThreads, key, val, cnt_s, sink, prune);
  }
}

// Rows with more than kBlockCap products: dense per-CTA accumulator slot.
template <typename T, typename LI, typename RI>
__global__ void __launch_bounds__(kDenseThreads)
spgemm_dense_kernel(const int *__restrict__ list, const int *__restrict__ count_ptr, const T *__restrict__ ld,
                    const LI *__restrict__ li, const LI *__restrict__ lp, const T *__restrict__ rd,
                    const RI *__restrict__ ri, const RI *__restrict__ rp, int64_t n_cols,
                    int *__restrict__ marker_base, float *__restrict__ accum_base, const int *__restrict__ flags,
                    RowSink<T> sink, bool prune) {
  __shared__ int wcnt[kDenseThreads / 32];
  if (*flags & 3) return;
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
    const int64_t out0 = sink.off[row];
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
      if (keep) {
        const int64_t pos = out0 + written + before + __popc(mask & ((1u << lane) - 1u));
        sink.col[pos] = (int)c;
        sink.val[pos] = v;
      }
      written += total;
      __syncthreads();
    }
    if (tid == 0) sink.row_nnz[row] = written;
    __syncthreads();
  }
}

// Copies every finished row from its upper-bound slot to its final place.
// One warp per row; lanes copy consecutive entries.
template <typename T, typename OutI>
__global__ void copy_rows_kernel(const int64_t *__restrict__ off, const int64_t *__restrict__ row_nnz,
                                 const int *__restrict__ col, const T *__restrict__ val, int64_t m,
                                 const OutI *__restrict__ out_indptr, OutI *__restrict__ out_idx,
                                 T *__restrict__ out_data) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t row = blockIdx.x * (int64_t)(blockDim.x >> 5) + (threadIdx.x >> 5); row < m; row += warps) {
    const int64_t n = row_nnz[row];
    const int64_t src = off[row], dst = (int64_t)out_indptr[row];
    for (int64_t j = lane; j < n; j += 32) {
      out_idx[dst + j] = (OutI)col[src + j];
      out_data[dst + j] = val[src + j];
    }
  }
}

template <typename OutI>
__global__ void widen_kernel(const int *__restrict__ col, int64_t n, OutI *__restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (OutI)col[i];
}

int dense_slots(int64_t n_cols) {
  const int64_t budget = (int64_t)256 << 20;
  int64_t slots = budget / std::max<int64_t>(n_cols * 8, 1);
  slots = std::max<int64_t>(1, std::min<int64_t>(slots, 2 * num_sms()));
  return (int)slots;
}

// Finished rows of one product (device memory from the stream-ordered pool).
struct Product {
  // what was multiplied
  const void *ptrs[6] = {};
  int64_t m = 0, rhs_rows = 0, n_cols = 0;
  int types[4] = {};
  bool prune = false;
  int device = -1;
  cudaStream_t stream = nullptr;
  // results
  void *mem = nullptr;
  int64_t *off = nullptr, *row_nnz = nullptr;
  int *col = nullptr;
  void *val = nullptr;
  int64_t nnz = 0;
  int64_t total_w = -1;  // products (the upper-bound layout's length)
  ~Product() {
    if (mem) cudaFreeAsync(mem, stream);
  }
  bool same(const Product &o) const {
    for (int i = 0; i < 6; ++i)
      if (ptrs[i] != o.ptrs[i]) return false;
    for (int i = 0; i < 4; ++i)
      if (types[i] != o.types[i]) return false;
    return m == o.m && rhs_rows == o.rhs_rows && n_cols == o.n_cols && prune == o.prune && device == o.device &&
           stream == o.stream;
  }
};

// The finished rows of this thread's last symbolic call, for its numeric call.
thread_local std::unique_ptr<Product> g_last_product;

// Expands, sorts and sums every row into a new Product; synchronises `s`
// twice (total product count, output nnz) and validates the indices.
template <typename T, typename LI, typename RI, typename OutI>
std::unique_ptr<Product> compute_product(std::unique_ptr<Product> P, const T *ld, const LI *li, const LI *lp,
                                         const T *rd, const RI *ri, const RI *rp, OutI *out_indptr,
                                         cudaStream_t s) {
  const int64_t m = P->m, rhs_rows = P->rhs_rows, n_cols = P->n_cols;
  const bool prune = P->prune;
  const int slots = dense_slots(n_cols);
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  const int64_t n_sums = scan_scratch_elems(m);
  size_t off = 0;
  const size_t o_work = off; off += al(sizeof(int64_t) * m);
  const size_t o_lists = off; off += al(sizeof(int) * kBins * m);
  const size_t o_counts = off; off += al(sizeof(int) * (kBins + 1));
  const size_t o_sums = off; off += al(sizeof(int64_t) * n_sums);
  Scratch scratch(off, s);
  char *base = scratch.as<char>();
  int64_t *work = reinterpret_cast<int64_t *>(base + o_work);
  int *lists = reinterpret_cast<int *>(base + o_lists);
  int *counts = reinterpret_cast<int *>(base + o_counts);  // [0..kBins) bins, [kBins] flags
  int64_t *sums = reinterpret_cast<int64_t *>(base + o_sums);
  int *flags = counts + kBins;

  // the product's own memory: offsets (m + 1), exact counts (m), then the
  // rows' columns and values at the offsets (sized after the first sync)
  MSX_CUDA(cudaMemsetAsync(counts, 0, sizeof(int) * (kBins + 1), s));
  const int t = 256;
  size_t head = al(sizeof(int64_t) * (m + 1)) + al(sizeof(int64_t) * m);
  Scratch head_mem(head, s);
  int64_t *row_off = head_mem.as<int64_t>();
  int64_t *row_nnz = reinterpret_cast<int64_t *>(head_mem.as<char>() + al(sizeof(int64_t) * (m + 1)));
  row_work_kernel<LI, RI><<<(unsigned)ceil_div(m, t), t, 0, s>>>(li, lp, rp, m, rhs_rows, work, flags);
  if (rhs_rows > 0)
    rhs_check_kernel<RI><<<(unsigned)ceil_div(rhs_rows, t), t, 0, s>>>(ri, rp, rhs_rows, n_cols, flags);
  // column << 8 | position fits 32 bits below the all-ones padding key
  const bool reg_ok = n_cols < ((int64_t)1 << 24);
  const bool quad_ok = reg_ok;
  bin_kernel<LI><<<(unsigned)ceil_div(m, t), t, 0, s>>>(work, lp, m, reg_ok, quad_ok, lists, counts, row_nnz);
  MSX_CHECK_LAUNCH();
  scan_counts_to_indptr<int64_t>(work, m, row_off, sums, s);
  struct {
    int counts[kBins + 1];
    int64_t total;
  } h{};
  MSX_CUDA(cudaMemcpyAsync(h.counts, counts, sizeof(h.counts), cudaMemcpyDeviceToHost, s));
  MSX_CUDA(cudaMemcpyAsync(&h.total, sums + n_sums - 1, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
  MSX_CUDA(cudaStreamSynchronize(s));
  if (h.counts[kBins] & 1) fail(MSX_ERR_INVALID, "csr_matmat lhs indices contain an out-of-bounds column.");
  if (h.counts[kBins] & 2) fail(MSX_ERR_INVALID, "csr_matmat rhs indices contain an out-of-bounds column.");
  const int64_t total = h.total;
  P->total_w = total;

  const size_t o_col = 0;
  size_t bytes = al(sizeof(int) * std::max<int64_t>(total, 1));
  const size_t o_val = bytes;
  bytes += al(sizeof(T) * std::max<int64_t>(total, 1));
  const size_t o_head = bytes;
  bytes += head;
  MSX_CUDA(cudaMallocAsync(&P->mem, bytes, s));
  char *pm = static_cast<char *>(P->mem);
  P->col = reinterpret_cast<int *>(pm + o_col);
  P->val = pm + o_val;
  P->off = reinterpret_cast<int64_t *>(pm + o_head);
  P->row_nnz = reinterpret_cast<int64_t *>(pm + o_head + al(sizeof(int64_t) * (m + 1)));
  MSX_CUDA(cudaMemcpyAsync(P->off, row_off, head, cudaMemcpyDeviceToDevice, s));
  RowSink<T> sink{P->off, P->col, static_cast<T *>(P->val), P->row_nnz};

  const int sms = num_sms();
  if (h.counts[0] > 0) {
    const int wpb = kBlockThreads / 32;
    const int grid = (int)std::min<int64_t>(ceil_div(h.counts[0], wpb), (int64_t)sms * 8);
    spgemm_warp_kernel<T, LI, RI><<<grid, kBlockThreads, 0, s>>>(lists, counts + 0, flags, ld, li, lp, rd, ri, rp,
                                                                  sink, prune);
    MSX_CHECK_LAUNCH();
  }
  auto reg_rows = [&](auto rtag) {
    constexpr int R = decltype(rtag)::value;
    constexpr int b = R == 1 ? 3 : (R == 2 ? 4 : (R == 4 ? 5 : 6));
    if (h.counts[b] == 0) return;
    const int wpb = kBlockThreads / 32;
    const int grid = (int)std::min<int64_t>(ceil_div(h.counts[b], wpb), (int64_t)sms * 8);
    spgemm_warp_reg_kernel<T, LI, RI, R><<<grid, kBlockThreads, 0, s>>>(lists + b * m, counts + b, flags, work, ld,
                                                                         li, lp, rd, ri, rp, sink, prune);
    MSX_CHECK_LAUNCH();
  };
  if (h.counts[7] > 0) {
    const int wpb = kBlockThreads / 32;
    const int grid = (int)std::min<int64_t>(ceil_div(ceil_div(h.counts[7], 4), wpb), (int64_t)sms * 8);
    spgemm_quad_kernel<T, LI, RI><<<grid, kBlockThreads, 0, s>>>(lists + 7 * m, counts + 7, flags, work, ld, li, lp,
                                                                  rd, ri, rp, sink, prune);
    MSX_CHECK_LAUNCH();
  }
  reg_rows(std::integral_constant<int, 1>{});
  reg_rows(std::integral_constant<int, 2>{});
  reg_rows(std::integral_constant<int, 4>{});
  reg_rows(std::integral_constant<int, 8>{});
  if (h.counts[1] > 0) {
    const size_t smem = (size_t)kBlockCap * (sizeof(uint64_t) + sizeof(float));
    const int grid = (int)std::min<int64_t>(h.counts[1], (int64_t)sms * 4);
    auto kern = spgemm_block_kernel<T, LI, RI>;
    MSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<grid, kBlockThreads, smem, s>>>(lists + m, counts + 1, flags, ld, li, lp, rd, ri, rp, sink, prune);
    MSX_CHECK_LAUNCH();
  }
  if (h.counts[2] > 0) {
    Scratch dense((sizeof(int) + sizeof(float)) * (size_t)slots * n_cols, s);
    int *marker = dense.as<int>();
    float *accum = reinterpret_cast<float *>(marker + (size_t)slots * n_cols);
    MSX_CUDA(cudaMemsetAsync(marker, 0xff, sizeof(int) * (size_t)slots * n_cols, s));
    const int grid = std::min(h.counts[2], slots);
    spgemm_dense_kernel<T, LI, RI><<<grid, kDenseThreads, 0, s>>>(lists + 2 * m, counts + 2, ld, li, lp, rd, ri, rp,
                                                                   n_cols, marker, accum, flags, sink, prune);
    MSX_CHECK_LAUNCH();
  }
  if (out_indptr) {
    scan_counts_to_indptr<OutI>(P->row_nnz, m, out_indptr, sums, s);
    MSX_CUDA(cudaMemcpyAsync(&P->nnz, sums + n_sums - 1, sizeof(int64_t), cudaMemcpyDeviceToHost, s));
    MSX_CUDA(cudaStreamSynchronize(s));
  }
  return P;
}

template <typename T, typename LI, typename RI, typename OutI>
void spgemm_pass(bool write, const T *ld, const LI *li, const LI *lp, const T *rd, const RI *ri, const RI *rp,
                 int64_t m, int64_t rhs_rows, int64_t n_cols, const int types[4], OutI *out_indptr, OutI *out_idx,
                 T *out_data, int64_t *out_nnz, bool prune, cudaStream_t s) {
  // numeric call: *out_nnz is the capacity of the caller's arrays
  const int64_t out_nnz_cap = write ? *out_nnz : 0;
  if (m == 0) {
    if (!write) {
      MSX_CUDA(cudaMemsetAsync(out_indptr, 0, sizeof(OutI), s));
      MSX_CUDA(cudaStreamSynchronize(s));
      *out_nnz = 0;
    }
    return;
  }
  auto key = std::make_unique<Product>();
  const void *ptrs[6] = {ld, li, lp, rd, ri, rp};
  for (int i = 0; i < 6; ++i) key->ptrs[i] = ptrs[i];
  for (int i = 0; i < 4; ++i) key->types[i] = types[i];
  key->m = m;
  key->rhs_rows = rhs_rows;
  key->n_cols = n_cols;
  key->prune = prune;
  key->stream = s;
  MSX_CUDA(cudaGetDevice(&key->device));
  if (!write) {
    g_last_product.reset();
    auto P = compute_product<T, LI, RI, OutI>(std::move(key), ld, li, lp, rd, ri, rp, out_indptr, s);
    const int64_t total = P->nnz;
    if (total > (int64_t)INT32_MAX) fail(MSX_ERR_OVERFLOW, "csr_matmat output nnz exceeds MLX shape limits.");
    if (sizeof(OutI) == 4 && total > (int64_t)INT32_MAX)
      fail(MSX_ERR_OVERFLOW, "csr_matmat output nnz exceeds index dtype capacity.");
    *out_nnz = total;
    g_last_product = std::move(P);
    return;
  }
  std::unique_ptr<Product> P;
  if (g_last_product && g_last_product->same(*key)) {
    P = std::move(g_last_product);
  } else {
    // not the product the last symbolic call computed: recompute its rows
    // (the caller's indptr already holds the output layout)
    P = compute_product<T, LI, RI, OutI>(std::move(key), ld, li, lp, rd, ri, rp, nullptr, s);
  }
  if (P->nnz == P->total_w && P->nnz >= 0 && P->nnz <= out_nnz_cap) {
    // no row lost an entry (no repeated columns, nothing pruned): the upper-
    // bound layout is already the packed output
    const int64_t n = P->nnz;
    if (n > 0) {
      MSX_CUDA(cudaMemcpyAsync(out_data, P->val, sizeof(T) * (size_t)n, cudaMemcpyDeviceToDevice, s));
      if constexpr (sizeof(OutI) == sizeof(int)) {
        MSX_CUDA(cudaMemcpyAsync(out_idx, P->col, sizeof(int) * (size_t)n, cudaMemcpyDeviceToDevice, s));
      } else {
        widen_kernel<OutI><<<(unsigned)std::min<int64_t>(ceil_div(n, 256), (int64_t)num_sms() * 16), 256, 0, s>>>(
            P->col, n, out_idx);
        MSX_CHECK_LAUNCH();
      }
    }
    return;
  }
  const int grid = (int)std::min<int64_t>(ceil_div(m, 8), (int64_t)num_sms() * 16);
  copy_rows_kernel<T, OutI><<<grid, 256, 0, s>>>(P->off, P->row_nnz, P->col, static_cast<const T *>(P->val), m,
                                                 out_indptr, out_idx, out_data);
  MSX_CHECK_LAUNCH();
}

}  // namespace

void spgemm_run(bool write, int value_dtype, int lhs_it, const void *ld, const void *li, const void *lp, int rhs_it,
                const void *rd, const void *ri, const void *rp, int64_t m, int64_t rhs_rows, int64_t n_cols,
                int out_it, void *out_indptr, void *out_idx, void *out_data, int64_t *out_nnz, bool prune,
                cudaStream_t s) {
  const int types[4] = {value_dtype, lhs_it, rhs_it, out_it};
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
                                       n_cols, types, static_cast<OutI *>(out_indptr), static_cast<OutI *>(out_idx),
                                       static_cast<T *>(out_data), out_nnz, prune, s);
        });
      });
    });
  });
}

}  // namespace msx
