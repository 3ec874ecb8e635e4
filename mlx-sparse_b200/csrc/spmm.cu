// CSR x dense row-major matrix (SpMM) for sm_100a.
//
// Reference behaviour: src/sparse/csr_matmul/csr_matmul.cpp:83-222 - for each
// row, every nonzero adds data[p] * rhs[col[p], :] into a row accumulator (fp32
// for fp16/bf16 values), in nonzero order, then the row is cast and stored.
//
// B200 design: this is a gather of dense RHS rows, not a contraction, so it is
// bound by HBM/L2 bandwidth and uses no tensor cores. A group of L lanes owns
// one output row slab of W = L*V columns (V values per 16-byte vector per
// lane); each lane accumulates V columns sequentially over the row's
// nonzeros, which reproduces the reference's summation order exactly. The RHS
// columns are processed in slabs (grid.y) small enough that one slab of the
// RHS stays resident in L2 while all rows stream past it, so each random RHS
// row gather hits L2 instead of HBM; the matrix arrays are re-streamed once
// per slab with evict-first loads.
#include <algorithm>

#include "common.cuh"

namespace msx {

namespace {

// L2 eviction-priority policies: the RHS slab is gathered repeatedly and should
// stay resident (evict_last); the matrix arrays and the output are touched once
// per slab (evict_first).
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ float4 ld_v4_hint(const void *p, uint64_t pol) {
  float4 r;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
               : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w)
               : "l"(p), "l"(pol));
  return r;
}

template <typename T, int V>
__device__ __forceinline__ void load_vec(const T *p, float (&out)[V], uint64_t pol) {
  if constexpr (V * sizeof(T) == 16) {
    const float4 raw = ld_v4_hint(p, pol);
    const T *e = reinterpret_cast<const T *>(&raw);
#pragma unroll
    for (int i = 0; i < V; ++i) out[i] = VT<T>::load(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) out[i] = VT<T>::load(__ldg(p + i));
  }
}

template <typename T, int V>
__device__ __forceinline__ void store_vec(T *p, const float (&in)[V]) {
  if constexpr (V * sizeof(T) == 16) {
    float4 raw;
    T *e = reinterpret_cast<T *>(&raw);
#pragma unroll
    for (int i = 0; i < V; ++i) e[i] = VT<T>::store(in[i]);
    __stcs(reinterpret_cast<float4 *>(p), raw);
  } else {
#pragma unroll
    for (int i = 0; i < V; ++i) p[i] = VT<T>::store(in[i]);
  }
}

// grid.x: row blocks, grid.y: column slabs. A group of L lanes handles one row
// and W = L*V columns of slab blockIdx.y. The group loads up to L (index,
// value) pairs of its row with one coalesced load, then broadcasts them by
// shuffles and issues kUnroll independent RHS gathers per lane before
// accumulating, so each lane keeps several 16-byte gathers in flight. The
// nonzeros are still consumed strictly in order (the reference's order).
template <typename T, typename I, int V, int L, int kUnroll, int kMinBlocks, int kPairs = 1>
__global__ void __launch_bounds__(256, kMinBlocks)
spmm_kernel(const T *__restrict__ data, const I *__restrict__ indices, const I *__restrict__ indptr,
            const T *__restrict__ rhs, T *__restrict__ out, int64_t n_rows, int64_t k, int64_t slab_cols) {
  constexpr int kRowsPerBlock = 256 / L;
  const int lane = threadIdx.x & 31;
  const int lane_in_row = threadIdx.x % L;
  const unsigned gmask = (L == 32) ? 0xffffffffu : (((1u << L) - 1u) << (lane & ~(L - 1)));
  const int64_t row = blockIdx.x * (int64_t)kRowsPerBlock + threadIdx.x / L;
  const bool row_ok = row < n_rows;
  const int64_t slab0 = blockIdx.y * slab_cols;
  const int64_t slab1 = min(slab0 + slab_cols, k);
  const int64_t p0 = row_ok ? (int64_t)indptr[row] : 0;
  const int64_t p1 = row_ok ? (int64_t)indptr[row + 1] : 0;
  const uint64_t pol_rhs = policy_evict_last();
  for (int64_t c = slab0 + (int64_t)lane_in_row * V; c - (int64_t)lane_in_row * V < slab1; c += (int64_t)L * V) {
    const bool col_ok = c < slab1;
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
    for (int64_t base = p0; base < p1; base += (int64_t)L * kPairs) {
      // kPairs chunks of L (index, value) pairs loaded at once (one round trip)
      I my_col[kPairs];
      float my_val[kPairs];
#pragma unroll
      for (int pp = 0; pp < kPairs; ++pp) {
        const int64_t j = base + pp * L + lane_in_row;
        my_col[pp] = 0;
        my_val[pp] = 0.f;
        if (j < p1) {
          my_col[pp] = ld_stream(indices + j);
          my_val[pp] = VT<T>::load(ld_stream(data + j));
        }
      }
#pragma unroll
      for (int pp = 0; pp < kPairs; ++pp) {
        const int64_t cb = base + pp * L;
        if (cb >= p1) break;  // uniform within the group
        const int cnt = (int)min((int64_t)L, p1 - cb);
        for (int q = 0; q < cnt; q += kUnroll) {
          float a[kUnroll];
          float b[kUnroll][V];
#pragma unroll
          for (int u = 0; u < kUnroll; ++u) {
            const I col = __shfl_sync(gmask, my_col[pp], (q + u) & (L - 1), L);
            a[u] = __shfl_sync(gmask, my_val[pp], (q + u) & (L - 1), L);
            if (q + u < cnt && col_ok) load_vec<T, V>(rhs + (int64_t)col * k + c, b[u], pol_rhs);
          }
#pragma unroll
          for (int u = 0; u < kUnroll; ++u)
            if (q + u < cnt)
#pragma unroll
              for (int i = 0; i < V; ++i) acc[i] = add_rn(acc[i], mul_rn(a[u], b[u][i]));
        }
      }
    }
    if (row_ok && col_ok) store_vec<T, V>(out + row * k + c, acc);
  }
}

// Asynchronous-copy variant: the RHS gathers go to shared memory with 16-byte
// cp.async (L2-only, evict_last hint), so a gather in flight holds no
// registers and each thread keeps kDepth of them outstanding; every thread
// consumes only the slots it filled, in nonzero order, so no barrier is
// needed beyond the group's own pair staging. Same per-element order as the
// register kernel. Requires 16-byte vectors (V * sizeof(T) == 16).
constexpr int kAsyncChunk = 16;  // (index, value) pairs staged per row at a time

template <typename I, int L, int kDepth>
constexpr size_t spmm_async_smem() {
  return (size_t)kDepth * 256 * 16 + (size_t)(256 / L) * kAsyncChunk * (sizeof(I) + sizeof(float));
}

__device__ __forceinline__ void cp_async16_hint(void *dst, const void *src, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(dst)),
               "l"(src), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// acc0 += s * b0 and acc1 += s * b1, each as a round-to-nearest multiply
// followed by a round-to-nearest add (the reference's `acc += a * b` without
// contraction): both products with one packed f32x2 multiply (sm_100), the
// adds as scalar round-to-nearest adds.
__device__ __forceinline__ void mul_add_rn_x2(float &acc0, float &acc1, float s, float b0, float b1) {
  unsigned long long bb, ss, p;
  asm("mov.b64 %0, {%1, %2};" : "=l"(bb) : "f"(b0), "f"(b1));
  asm("mov.b64 %0, {%1, %1};" : "=l"(ss) : "f"(s));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(p) : "l"(ss), "l"(bb));
  float p0, p1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(p0), "=f"(p1) : "l"(p));
  acc0 = __fadd_rn(acc0, p0);
  acc1 = __fadd_rn(acc1, p1);
}

template <typename T, typename I, int V, int L, int kDepth>
__device__ __forceinline__ void spmm_async_block(const T *__restrict__ data, const I *__restrict__ indices,
                                                 const I *__restrict__ indptr, const T *__restrict__ rhs,
                                                 T *__restrict__ out, int64_t n_rows, int64_t k, int64_t slab_cols,
                                                 int64_t block_x, int64_t slab_y, unsigned char *spmm_sm) {
  static_assert(V * sizeof(T) == 16, "16-byte vectors only");
  constexpr int kRows = 256 / L;
  float4 *stage = reinterpret_cast<float4 *>(spmm_sm);  // [kDepth][256]
  I *col_s = reinterpret_cast<I *>(spmm_sm + (size_t)kDepth * 256 * 16);  // [kRows][kAsyncChunk]
  float *val_s = reinterpret_cast<float *>(col_s + kRows * kAsyncChunk);     // [kRows][kAsyncChunk]
  const int tid = threadIdx.x;
  const int lane = tid & 31;
  const int lane_in_row = tid % L;
  const int rloc = tid / L;
  const unsigned gmask = (L == 32) ? 0xffffffffu : (((1u << L) - 1u) << (lane & ~(L - 1)));
  const int64_t row = block_x * kRows + rloc;
  const bool row_ok = row < n_rows;
  const int64_t slab0 = slab_y * slab_cols;
  const int64_t slab1 = min(slab0 + slab_cols, k);
  const int64_t p0 = row_ok ? (int64_t)indptr[row] : 0;
  const int64_t p1 = row_ok ? (int64_t)indptr[row + 1] : 0;
  const uint64_t pol_rhs = policy_evict_last();
  I *my_cols = col_s + rloc * kAsyncChunk;
  float *my_vals = val_s + rloc * kAsyncChunk;
  for (int64_t c = slab0 + (int64_t)lane_in_row * V; c - (int64_t)lane_in_row * V < slab1; c += (int64_t)L * V) {
    const bool col_ok = c < slab1;
    float acc[V];
#pragma unroll
    for (int i = 0; i < V; ++i) acc[i] = 0.f;
    for (int64_t base = p0; base < p1; base += kAsyncChunk) {
      const int cnt = (int)min((int64_t)kAsyncChunk, p1 - base);
      __syncwarp(gmask);  // the previous chunk's pairs are no longer read
      for (int j = lane_in_row; j < cnt; j += L) {
        my_cols[j] = ld_stream(indices + base + j);
        my_vals[j] = VT<T>::load(ld_stream(data + base + j));
      }
      __syncwarp(gmask);
#pragma unroll
      for (int q = 0; q < kDepth; ++q) {
        if (q < cnt && col_ok) cp_async16_hint(&stage[q * 256 + tid], rhs + (int64_t)my_cols[q] * k + c, pol_rhs);
        cp_async_commit();
      }
      for (int q = 0; q < cnt; ++q) {
        cp_async_wait<kDepth - 1>();  // the group of gather q has landed
        const int slot = (q % kDepth) * 256 + tid;
        float b[V];
        if (col_ok) {
          const float4 raw = stage[slot];
          const T *e = reinterpret_cast<const T *>(&raw);
#pragma unroll
          for (int i = 0; i < V; ++i) b[i] = VT<T>::load(e[i]);
          const float a = my_vals[q];
#pragma unroll
          for (int i = 0; i < V; i += 2) mul_add_rn_x2(acc[i], acc[i + 1], a, b[i], b[i + 1]);
        }
        if (q + kDepth < cnt && col_ok)
          cp_async16_hint(&stage[slot], rhs + (int64_t)my_cols[q + kDepth] * k + c, pol_rhs);
        cp_async_commit();
      }
      cp_async_wait<0>();
    }
    if (row_ok && col_ok) store_vec<T, V>(out + row * k + c, acc);
  }
}

template <typename T, typename I, int V, int L, int kDepth>
__global__ void __launch_bounds__(256)
spmm_async_kernel(const T *__restrict__ data, const I *__restrict__ indices, const I *__restrict__ indptr,
                  const T *__restrict__ rhs, T *__restrict__ out, int64_t n_rows, int64_t k, int64_t slab_cols) {
  extern __shared__ __align__(16) unsigned char spmm_sm[];
  spmm_async_block<T, I, V, L, kDepth>(data, indices, indptr, rhs, out, n_rows, k, slab_cols, blockIdx.x, blockIdx.y,
                                       spmm_sm);
}

template <typename T, typename I, int V, int L, int kDepth>
void launch_spmm_async(dim3 grid, cudaStream_t stream, const T *data, const I *indices, const I *indptr,
                       const T *rhs, T *out, int64_t n_rows, int64_t k, int64_t slab_cols) {
  constexpr size_t smem = spmm_async_smem<I, L, kDepth>();
  static thread_local int configured_dev = -1;
  int dev = 0;
  MSX_CUDA(cudaGetDevice(&dev));
  if (dev != configured_dev) {
    MSX_CUDA(cudaFuncSetAttribute(spmm_async_kernel<T, I, V, L, kDepth>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    configured_dev = dev;
  }
  spmm_async_kernel<T, I, V, L, kDepth><<<grid, 256, smem, stream>>>(data, indices, indptr, rhs, out, n_rows, k,
                                                                    slab_cols);
}

template <typename T, typename I, int V, int L>
void launch_spmm(const T *data, const I *indices, const I *indptr, const T *rhs, T *out, int64_t n_rows,
                 int64_t k, int64_t slab_cols, cudaStream_t stream) {
  constexpr int kRowsPerBlock = 256 / L;
  const int64_t n_slabs = ceil_div(k, slab_cols);
  dim3 grid((unsigned)ceil_div(n_rows, kRowsPerBlock), (unsigned)n_slabs);
  // measured defaults: cp.async gathers 8 deep for 16-byte vectors (fp32
  // 0.555 ms vs 0.847, bf16 0.307 vs 0.800 ms on the 1M x 1M, 16/row, k = 64
  // config); else the register kernel with 8 gathers in flight at 4 CTAs/SM
  // for 4-byte values, 4 in flight at 6 CTAs/SM for 2-byte values
  if constexpr (V * sizeof(T) == 16) {
    launch_spmm_async<T, I, V, L, 8>(grid, stream, data, indices, indptr, rhs, out, n_rows, k, slab_cols);
  } else if constexpr (sizeof(T) == 2) {
    spmm_kernel<T, I, V, L, 4, 6, 2><<<grid, 256, 0, stream>>>(data, indices, indptr, rhs, out, n_rows, k, slab_cols);
  } else {
    spmm_kernel<T, I, V, L, 8, 4><<<grid, 256, 0, stream>>>(data, indices, indptr, rhs, out, n_rows, k, slab_cols);
  }
  MSX_CHECK_LAUNCH();
}

// Bytes per RHS row of one column slab: 256 (two 128-byte lines). On the
// 2^20 x 2^20, 16/row, k = 64 fp32 config a single 256-byte pass (matrix read
// once) measured 0.541 ms against 0.553 for two 128-byte slabs, 0.79 for 64;
// narrower slabs fit L2 better but the kernel is bound by gather issue
// (L1/TEX), not by DRAM misses. MSX_SPMM_SLAB_BYTES = 32/64/128/256 overrides.
int64_t spmm_slab_bytes(int64_t, int64_t) {
  if (const char *env = getenv("MSX_SPMM_SLAB_BYTES")) {
    const int64_t v = atoll(env);
    if (v == 32 || v == 64 || v == 128 || v == 256) return v;
  }
  return 256;
}

// Bytes of the RHS slab that should stay L2 resident while rows stream by.
int64_t spmm_l2_budget() {
  static int64_t budget = [] {
    const char *env = getenv("MSX_SPMM_L2_BYTES");
    if (env && *env) return (int64_t)atoll(env);
    int dev = 0, l2 = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, dev) == cudaSuccess && l2 > 0)
      return (int64_t)l2 * 3 / 4;
    return (int64_t)48 << 20;
  }();
  return budget;
}

}  // namespace

void spmm_run(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
              const void *rhs, int64_t k, void *out, int64_t n_rows, int64_t n_cols, int64_t nnz,
              cudaStream_t stream) {
  if (n_rows == 0 || k == 0) return;
  dispatch_value(value_dtype, [&](auto vtyp) {
    using T = decltype(vtyp);
    constexpr int kVec = 16 / sizeof(T);
    dispatch_index(index_dtype, [&](auto ityp) {
      using I = decltype(ityp);
      const bool vec_ok = (k % kVec == 0) && (reinterpret_cast<uintptr_t>(rhs) % 16 == 0) &&
                          (reinterpret_cast<uintptr_t>(out) % 16 == 0);
      const int64_t elem = sizeof(T);
      const T *d = static_cast<const T *>(data);
      const I *ix = static_cast<const I *>(indices);
      const I *ip = static_cast<const I *>(indptr);
      const T *b = static_cast<const T *>(rhs);
      T *o = static_cast<T *>(out);
      // One pass over the rows when the whole RHS fits the L2 budget (or the
      // env override forces it); otherwise column slabs whose RHS part fits
      // the budget (128, 64 or 32 bytes per RHS row), so the random row
      // gathers of a slab hit L2 while the matrix is re-streamed per slab.
      const int64_t budget = spmm_l2_budget();
      const int64_t slab_bytes = spmm_slab_bytes(n_cols, budget);
      const bool one_pass = n_cols * k * elem <= budget || k * elem <= slab_bytes;
      if (vec_ok) {
        const int64_t kv = k / kVec;  // 16-byte vectors per row
        const int64_t slab_vecs = one_pass ? kv : slab_bytes / 16;
        if (slab_vecs >= 16) {
          launch_spmm<T, I, kVec, 16>(d, ix, ip, b, o, n_rows, k, ceil_div(slab_vecs, 16) * 16 * kVec, stream);
        } else if (slab_vecs >= 8) {
          launch_spmm<T, I, kVec, 8>(d, ix, ip, b, o, n_rows, k, ceil_div(slab_vecs, 8) * 8 * kVec, stream);
        } else if (slab_vecs >= 4) {
          launch_spmm<T, I, kVec, 4>(d, ix, ip, b, o, n_rows, k, ceil_div(slab_vecs, 4) * 4 * kVec, stream);
        } else if (slab_vecs >= 2) {
          launch_spmm<T, I, kVec, 2>(d, ix, ip, b, o, n_rows, k, ceil_div(slab_vecs, 2) * 2 * kVec, stream);
        } else {
          launch_spmm<T, I, kVec, 1>(d, ix, ip, b, o, n_rows, k, kVec, stream);
        }
      } else {
        // Scalar path for widths that are not a multiple of the 16-byte vector.
        if (k >= 16) {
          launch_spmm<T, I, 1, 16>(d, ix, ip, b, o, n_rows, k, one_pass ? ceil_div(k, 16) * 16 : 32, stream);
        } else if (k >= 4) {
          launch_spmm<T, I, 1, 4>(d, ix, ip, b, o, n_rows, k, k, stream);
        } else {
          launch_spmm<T, I, 1, 1>(d, ix, ip, b, o, n_rows, k, k, stream);
        }
      }
    });
  });
}

}  // namespace msx
