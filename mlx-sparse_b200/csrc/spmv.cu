// CSR SpMV (y = A x) for sm_100a.
//
// Reference behaviour: src/sparse/csr_matvec/csr_matvec.cpp:79-168 - every row
// is a sequential fp32 (or fp32-accumulated fp16/bf16) sum of data[p]*x[col[p]],
// rows are independent, and the CPU path splits rows into nnz-weighted worker
// ranges (src/common/cpu_parallel.cpp:202-253).
//
// B200 design: the matrix is cut into row-aligned merge-path tiles of about
// kTileItems path items (rows + nonzeros), so every tile streams about the same
// number of bytes whatever the row-length distribution. A persistent grid (a
// few CTAs per SM) walks the tiles; each CTA double-buffers them in shared
// memory with TMA bulk copies (spmv.cuh). Inside a tile the products
// data*x[col] are formed with every gather in flight at once, then each row is
// summed from shared memory: by one thread, left to right as the reference
// does, for rows of up to 32 nonzeros, by a warp for longer rows. Rows longer
// than kSplitRowLen are split between tiles; their tile partials go to scratch
// and a small fixup kernel adds them in tile order (deterministic, no
// atomics on values).
#include <atomic>

#include "spmv.cuh"

namespace msx {

namespace {

template <typename I>
__global__ void spmv_plan_kernel(const I *__restrict__ indptr, int64_t n_rows, int64_t nnz, int64_t n_tiles,
                                 int64_t *__restrict__ tile_row, int64_t *__restrict__ tile_nz,
                                 unsigned long long *__restrict__ n_split) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t > n_tiles) return;
  const int64_t total = n_rows + nnz;
  int64_t diag = t * (int64_t)kTileItems;
  if (diag > total || t == n_tiles) diag = total;
  const int64_t r = merge_path_search(diag, n_rows, nnz, [&](int64_t i) { return (int64_t)indptr[i + 1]; });
  int64_t k = diag - r;
  if (r < n_rows) {
    const int64_t start = (int64_t)indptr[r];
    if (k > start) {
      const int64_t len = (int64_t)indptr[r + 1] - start;
      if (len <= kSplitRowLen) {
        k = start;  // snap to the row start: short rows never cross tiles
      } else {
        atomicAdd(n_split, 1ull);
      }
    }
  }
  tile_row[t] = r;
  tile_nz[t] = k;
}

// Adds the tile partials of split rows in tile order. One thread per tile; the
// first tile touching a split row walks forward over the tiles it spans.
template <typename T, typename I>
__global__ void spmv_fixup_kernel(const I *__restrict__ indptr, T *__restrict__ y,
                                  const int64_t *__restrict__ tile_row, const int64_t *__restrict__ tile_nz,
                                  const float *__restrict__ carry_head, const float *__restrict__ carry_tail,
                                  int64_t n_tiles) {
  const int64_t t = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (t >= n_tiles) return;
  const int64_t row = tile_row[t + 1];
  const int64_t row_start = (int64_t)indptr[row];
  // Only tiles that end inside row `row` ...
  if (!(tile_nz[t + 1] > row_start)) return;
  // ... and are the first tile of that row (they did not begin inside it).
  if (tile_row[t] == row && tile_nz[t] > row_start) return;
  float sum = carry_tail[t];
  int64_t u = t + 1;
  // Tiles lying wholly inside the row finish no row: tile_row[u+1] == row.
  while (u < n_tiles && tile_row[u + 1] == row) {
    sum = add_rn(sum, carry_tail[u]);
    ++u;
  }
  // Tile u finishes the row; its head partial comes last.
  if (u < n_tiles) sum = add_rn(sum, carry_head[u]);
  y[row] = VT<T>::store(sum);
}

}  // namespace

int64_t spmv_num_tiles(int64_t n_rows, int64_t nnz) {
  const int64_t total = n_rows + nnz;
  return total == 0 ? 0 : ceil_div(total, kTileItems);
}

size_t spmv_plan_device_bytes(int64_t n_tiles) {
  // split counter (16 B), tile_row[n+1], tile_nz[n+1]
  return 16 + sizeof(int64_t) * 2 * (n_tiles + 1);
}

void spmv_plan_layout(void *base, int64_t n_tiles, int64_t **tile_row, int64_t **tile_nz,
                      unsigned long long **n_split) {
  char *p = static_cast<char *>(base);
  *n_split = reinterpret_cast<unsigned long long *>(p);
  *tile_row = reinterpret_cast<int64_t *>(p + 16);
  *tile_nz = *tile_row + (n_tiles + 1);
}

void spmv_build_plan(int index_dtype, const void *indptr, int64_t n_rows, int64_t nnz, void *plan_dev,
                     int64_t n_tiles, cudaStream_t stream) {
  int64_t *tile_row, *tile_nz;
  unsigned long long *n_split;
  spmv_plan_layout(plan_dev, n_tiles, &tile_row, &tile_nz, &n_split);
  MSX_CUDA(cudaMemsetAsync(n_split, 0, sizeof(unsigned long long), stream));
  if (n_tiles == 0) return;
  const int threads = 256;
  const int64_t blocks = ceil_div(n_tiles + 1, threads);
  dispatch_index(index_dtype, [&](auto ityp) {
    using I = decltype(ityp);
    spmv_plan_kernel<I><<<(unsigned)blocks, threads, 0, stream>>>(static_cast<const I *>(indptr), n_rows, nnz,
                                                                 n_tiles, tile_row, tile_nz, n_split);
  });
  MSX_CHECK_LAUNCH();
}

namespace {
__device__ int g_spmv_error;
std::atomic<long long> g_poll_limit{kMaxPolls};
}  // namespace

// Looked up on every call (cheap), so the address is right for whatever
// context is current, including after a device reset.
int *spmv_error_flag() {
  int *ptr = nullptr;
  MSX_CUDA(cudaGetSymbolAddress(reinterpret_cast<void **>(&ptr), g_spmv_error));
  return ptr;
}

long long spmv_poll_limit() { return g_poll_limit.load(std::memory_order_relaxed); }
void spmv_set_poll_limit(long long v) { g_poll_limit.store(v < 0 ? kMaxPolls : v, std::memory_order_relaxed); }

// Reads and clears this device's SpMV timeout flag.
bool spmv_take_error() {
  int v = 0;
  MSX_CUDA(cudaMemcpyFromSymbol(&v, g_spmv_error, sizeof(int)));
  if (v) {
    const int zero = 0;
    MSX_CUDA(cudaMemcpyToSymbol(g_spmv_error, &zero, sizeof(int)));
  }
  return v != 0;
}

// The TMA bulk-copy pipeline of the tile kernel is opt-in (MSX_SPMV_TMA=1,
// read at every call): plain loads measured faster on B200 (Lap2D 1024^2
// 46 us against 57, 2^22-row power-law 0.565 ms against 1.078).
bool spmv_tma_ok(const void *data, const void *indices, const void *indptr) {
  const char *e = getenv("MSX_SPMV_TMA");
  const bool enabled = e && *e && *e != '0';
  auto al = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  return enabled && al(data) && al(indices) && al(indptr);
}

int spmv_grid(int64_t n_tiles) { return spmv_grid_for<float, int32_t, NoEpilogue>(n_tiles, true); }

void spmv_run(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
              const void *x, void *y, int64_t n_rows, int64_t nnz, const void *plan_dev, int64_t n_tiles,
              bool launch_fixup, float *carry_scratch, cudaStream_t stream) {
  if (n_tiles == 0) return;
  int64_t *tile_row, *tile_nz;
  unsigned long long *n_split;
  spmv_plan_layout(const_cast<void *>(plan_dev), n_tiles, &tile_row, &tile_nz, &n_split);
  float *carry_head = carry_scratch;
  float *carry_tail = carry_scratch ? carry_scratch + n_tiles : nullptr;
  dispatch_value(value_dtype, [&](auto vtyp) {
    using T = decltype(vtyp);
    dispatch_index(index_dtype, [&](auto ityp) {
      using I = decltype(ityp);
      launch_spmv_tiles<T, I, NoEpilogue>(static_cast<const T *>(data), static_cast<const I *>(indices),
                                          static_cast<const I *>(indptr), static_cast<const T *>(x),
                                          static_cast<T *>(y), tile_row, tile_nz, carry_head, carry_tail, n_tiles,
                                          nnz, n_rows, NoEpilogue{}, stream);
      if (launch_fixup) {
        const int threads = 256;
        spmv_fixup_kernel<T, I><<<(unsigned)ceil_div(n_tiles, threads), threads, 0, stream>>>(
            static_cast<const I *>(indptr), static_cast<T *>(y), tile_row, tile_nz, carry_head, carry_tail,
            n_tiles);
        MSX_CHECK_LAUNCH();
      }
    });
  });
}

void spmv_fixup_f32(int index_dtype, const void *indptr, float *y, const void *plan_dev, int64_t n_tiles,
                    const float *carry_scratch, cudaStream_t stream) {
  if (n_tiles == 0) return;
  int64_t *tile_row, *tile_nz;
  unsigned long long *n_split;
  spmv_plan_layout(const_cast<void *>(plan_dev), n_tiles, &tile_row, &tile_nz, &n_split);
  const int threads = 256;
  dispatch_index(index_dtype, [&](auto ityp) {
    using I = decltype(ityp);
    spmv_fixup_kernel<float, I><<<(unsigned)ceil_div(n_tiles, threads), threads, 0, stream>>>(
        static_cast<const I *>(indptr), y, tile_row, tile_nz, carry_scratch, carry_scratch + n_tiles, n_tiles);
  });
  MSX_CHECK_LAUNCH();
}

}  // namespace msx

// ---- diagonal extraction (setup of Jacobi preconditioners) ------------------
namespace msx {
namespace {
template <typename T, typename I>
__global__ void csr_diagonal_kernel(const T *__restrict__ data, const I *__restrict__ indices,
                                    const I *__restrict__ indptr, int64_t n_diag, T *__restrict__ out) {
  const int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (r >= n_diag) return;
  float acc = 0.f;  // duplicates of the diagonal entry summed in stored order
  for (int64_t p = (int64_t)indptr[r]; p < (int64_t)indptr[r + 1]; ++p)
    if ((int64_t)indices[p] == r) acc = add_rn(acc, VT<T>::load(data[p]));
  out[r] = VT<T>::store(acc);
}
}  // namespace

void csr_diagonal_run(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
                      int64_t n_diag, void *out, cudaStream_t stream) {
  if (n_diag == 0) return;
  dispatch_value(value_dtype, [&](auto vt) {
    using T = decltype(vt);
    dispatch_index(index_dtype, [&](auto it) {
      using I = decltype(it);
      csr_diagonal_kernel<T, I><<<(unsigned)ceil_div(n_diag, 256), 256, 0, stream>>>(
          static_cast<const T *>(data), static_cast<const I *>(indices), static_cast<const I *>(indptr), n_diag,
          static_cast<T *>(out));
    });
  });
  MSX_CHECK_LAUNCH();
}
}  // namespace msx
