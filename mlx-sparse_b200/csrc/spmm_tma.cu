// SpMM with TMA row gathers (tile::gather4) for sm_100a.
//
// Same product and summation order as spmm.cu (the reference's
// src/sparse/csr_matmul/csr_matmul.cpp:83-222: each output element is the
// in-order sum over the row's nonzeros of data[p] * rhs[col[p], c]), but the
// random RHS rows are fetched by the Tensor Memory Accelerator instead of by
// thread loads: in a persistent CTA one producer warp cuts the CTA's rows into
// row-aligned stages of at most kSlots nonzeros, and for every four nonzeros
// issues one `cp.async.bulk.tensor.2d ... tile::gather4` that copies four
// whole RHS rows (one 128- or 256-byte box row each) into shared memory,
// completing on the stage's mbarrier. Eight consumer warps wait on the stage,
// and a group of 16-byte lanes per output row multiplies the staged RHS rows by
// the row's values in nonzero order, then releases the stage. With four
// stages per CTA the TMA keeps several stages of gathers in flight while
// another is consumed, independently of register pressure.
//
// Rows with more than kSlots nonzeros are skipped here and finished by the
// register kernel (spmm.cu) restricted to them. TMA rules observed: the
// tensor map covers only this GPU's B (no multicast anywhere), boxes are one
// row high, the inner coordinate is a multiple of 16 bytes, and every mbarrier
// wait is bounded (timeouts set an error flag and end the kernel).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace msx {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kStages = 4;
constexpr int kSlots = 128;  // gathered RHS rows per stage
constexpr long long kPollLimit = 1ll << 22;

struct StageDesc {
  long long row0;
  long long k0;
  int nrows;
  int nnz;
  int flags;  // 1: done, 2: single row too long for a stage (skipped)
  int pad;
};

__device__ int g_spmm_tma_error;

__device__ __forceinline__ uint32_t sptr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint64_t *b, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sptr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t *b) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sptr(b)) : "memory");
}
__device__ __forceinline__ void bar_arrive_tx(uint64_t *b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sptr(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool bar_try_wait(uint64_t *b, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(sptr(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; false after kPollLimit polls (error flagged).
__device__ __forceinline__ bool bar_wait(uint64_t *b, uint32_t parity) {
  long long polls = 0;
  while (!bar_try_wait(b, parity)) {
    if (++polls > kPollLimit) {
      atomicOr(&g_spmm_tma_error, 1);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void gather4(void *dst, const CUtensorMap *map, uint64_t *bar, int x, int r0, int r1,
                                        int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(sptr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(sptr(bar)), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3)
      : "memory");
}

template <typename T, typename I, int V, int G>
__global__ void __launch_bounds__(kThreads, 1)
spmm_tma_kernel(const __grid_constant__ CUtensorMap map, const T *__restrict__ data, const I *__restrict__ indices,
                const I *__restrict__ indptr, T *__restrict__ out, int64_t n_rows, int64_t nnz, int64_t k,
                int slab_cols) {
  // G lanes x 16 bytes = one box row of slab_cols values.
  constexpr int kBoxBytes = G * 16;
  constexpr int kRowsPerStage = (kConsumerWarps * 32) / G;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // TMA destinations start on a 1024-byte boundary (1 KB of slack is allocated)
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char *stage_buf = smem;  // kStages * kSlots * kBoxBytes
  StageDesc *desc = reinterpret_cast<StageDesc *>(smem + (size_t)kStages * kSlots * kBoxBytes);
  uint64_t *full = reinterpret_cast<uint64_t *>(desc + kStages);
  uint64_t *empty = full + kStages;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int col0 = blockIdx.y * slab_cols;
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], kConsumerWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    // ---------------- producer warp ----------------
    // nnz-balanced contiguous row range of this CTA
    auto row_at = [&](int64_t target) {
      int64_t lo = 0, hi = n_rows;
      while (lo < hi) {
        const int64_t mid = (lo + hi) >> 1;
        if ((int64_t)indptr[mid] < target) lo = mid + 1;
        else hi = mid;
      }
      return lo;
    };
    const int64_t rb = blockIdx.x == 0 ? 0 : row_at(nnz * (int64_t)blockIdx.x / gridDim.x);
    const int64_t re = blockIdx.x + 1 == gridDim.x ? n_rows : row_at(nnz * (int64_t)(blockIdx.x + 1) / gridDim.x);
    int64_t row = rb;
    for (int j = 0;; ++j) {
      const int s = j % kStages;
      if (j >= kStages && !bar_wait(&empty[s], (uint32_t)((j / kStages - 1) & 1))) return;
      StageDesc d{};
      if (lane == 0) {
        d.row0 = row;
        d.k0 = row < re ? (int64_t)indptr[row] : 0;
        if (row >= re) {
          d.flags = 1;
        } else {
          int64_t r = row;
          int cnt = 0;
          while (r < re && d.nrows < kRowsPerStage) {
            const int64_t len = (int64_t)indptr[r + 1] - (int64_t)indptr[r];
            if (len > kSlots) {
              if (d.nrows == 0) {  // a lone long row: skipped here
                d.nrows = 1;
                d.flags = 2;
                r = r + 1;
              }
              break;
            }
            if (cnt + len > kSlots) break;
            cnt += (int)len;
            ++d.nrows;
            ++r;
          }
          d.nnz = d.flags == 2 ? 0 : cnt;
        }
        desc[s] = d;
      }
      d.row0 = __shfl_sync(0xffffffffu, d.row0, 0);
      d.k0 = __shfl_sync(0xffffffffu, d.k0, 0);
      d.nrows = __shfl_sync(0xffffffffu, d.nrows, 0);
      d.nnz = __shfl_sync(0xffffffffu, d.nnz, 0);
      d.flags = __shfl_sync(0xffffffffu, d.flags, 0);
      const int groups = (d.nnz + 3) / 4;
      if (lane == 0) bar_arrive_tx(&full[s], (uint32_t)(groups * 4 * kBoxBytes));
      __syncwarp();
      unsigned char *buf = stage_buf + (size_t)s * kSlots * kBoxBytes;
      for (int g = lane; g < groups; g += 32) {
        int c[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int q = min(4 * g + t, d.nnz - 1);  // pad with a repeat of the last row
          c[t] = (int)indices[d.k0 + q];
        }
        gather4(buf + (size_t)g * 4 * kBoxBytes, &map, &full[s], col0, c[0], c[1], c[2], c[3]);
      }
      if (d.flags & 1) return;
      row += d.nrows;
    }
  }

  // ---------------- consumer warps ----------------
  const int grp = tid / G, lane_g = tid % G;
  for (int j = 0;; ++j) {
    const int s = j % kStages;
    if (!bar_wait(&full[s], (uint32_t)((j / kStages) & 1))) return;
    const StageDesc d = desc[s];
    if (d.flags & 1) break;
    if (!(d.flags & 2) && grp < d.nrows) {
      const int64_t row = d.row0 + grp;
      const int64_t p0 = (int64_t)indptr[row], p1 = (int64_t)indptr[row + 1];
      const unsigned char *buf = stage_buf + (size_t)s * kSlots * kBoxBytes;
      float acc[V];
#pragma unroll
      for (int i = 0; i < V; ++i) acc[i] = 0.f;
      const unsigned gmask = (G == 32) ? 0xffffffffu : (((1u << G) - 1u) << (lane & ~(G - 1)));
      for (int64_t base = p0; base < p1; base += G) {
        // one coalesced load of up to G values, broadcast by shuffles
        const float my_val = base + lane_g < p1 ? VT<T>::load(__ldg(data + base + lane_g)) : 0.f;
        const int cnt = (int)min((int64_t)G, p1 - base);
        const unsigned char *src = buf + (size_t)(base - d.k0) * kBoxBytes + (size_t)lane_g * 16;
        for (int q = 0; q < cnt; ++q) {
          const float a = __shfl_sync(gmask, my_val, q, G);
          const float4 raw = *reinterpret_cast<const float4 *>(src + (size_t)q * kBoxBytes);
          const T *e = reinterpret_cast<const T *>(&raw);
#pragma unroll
          for (int i = 0; i < V; ++i) acc[i] = add_rn(acc[i], mul_rn(a, VT<T>::load(e[i])));
        }
      }
      const int64_t c = (int64_t)col0 + (int64_t)lane_g * V;
      if (c < k) {
        float4 o;
        T *oe = reinterpret_cast<T *>(&o);
#pragma unroll
        for (int i = 0; i < V; ++i) oe[i] = VT<T>::store(acc[i]);
        __stcs(reinterpret_cast<float4 *>(out + row * k + c), o);
      }
    }
    __syncwarp();
    if (lane == 0) bar_arrive(&empty[s]);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

template <typename T> CUtensorMapDataType tma_type();
template <> CUtensorMapDataType tma_type<float>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT32; }
template <> CUtensorMapDataType tma_type<__half>() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT16; }
template <> CUtensorMapDataType tma_type<__nv_bfloat16>() { return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16; }

template <typename T, typename I, int G>
bool launch_tma(const T *data, const I *indices, const I *indptr, const T *rhs, T *out, int64_t n_rows,
                int64_t n_cols, int64_t nnz, int64_t k, cudaStream_t stream) {
  constexpr int V = 16 / sizeof(T);
  constexpr int kBoxBytes = G * 16;
  const int slab_cols = kBoxBytes / (int)sizeof(T);
  auto fn = encode_fn();
  if (!fn) return false;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)n_cols};
  cuuint64_t strides[1] = {(cuuint64_t)(k * sizeof(T))};
  cuuint32_t box[2] = {(cuuint32_t)slab_cols, 1};
  cuuint32_t estr[2] = {1, 1};
  if (fn(&map, tma_type<T>(), 2, const_cast<T *>(rhs), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  const size_t smem = 1024 + (size_t)kStages * kSlots * kBoxBytes + kStages * sizeof(StageDesc) + 2 * kStages * 8;
  auto kern = spmm_tma_kernel<T, I, V, G>;
  MSX_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  int occ = 0;
  MSX_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kThreads, smem));
  const int64_t grid_x = std::max<int64_t>(1, std::min<int64_t>((int64_t)std::max(occ, 1) * num_sms(), n_rows));
  dim3 grid((unsigned)grid_x, (unsigned)ceil_div(k, slab_cols));
  kern<<<grid, kThreads, smem, stream>>>(map, data, indices, indptr, out, n_rows, nnz, k, slab_cols);
  MSX_CHECK_LAUNCH();
  return true;
}

}  // namespace

// Rows longer than this are left to the register kernel.
int64_t spmm_tma_max_row() { return kSlots; }

// Returns false (nothing launched) when the TMA path does not apply.
bool spmm_tma_run(int value_dtype, int index_dtype, const void *data, const void *indices, const void *indptr,
                  const void *rhs, int64_t k, void *out, int64_t n_rows, int64_t n_cols, int64_t nnz,
                  cudaStream_t stream) {
  static const int mode = [] {
    // opt-in: on the SpMM configs measured so far the register kernel is
    // faster (TMA gathers are issue-rate bound at one CTA per SM)
    const char *e = getenv("MSX_SPMM_TMA");
    return e && *e ? atoi(e) : 0;
  }();
  if (!mode || n_rows == 0 || nnz == 0 || n_cols > INT32_MAX) return false;
  bool ok = false;
  dispatch_value(value_dtype, [&](auto vt) {
    using T = decltype(vt);
    const int64_t row_bytes = k * (int64_t)sizeof(T);
    // whole 128- or 256-byte box rows, 16-byte aligned bases
    if ((reinterpret_cast<uintptr_t>(rhs) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return;
    dispatch_index(index_dtype, [&](auto it) {
      using I = decltype(it);
      if (row_bytes % 256 == 0)
        ok = launch_tma<T, I, 16>(static_cast<const T *>(data), static_cast<const I *>(indices),
                                  static_cast<const I *>(indptr), static_cast<const T *>(rhs), static_cast<T *>(out),
                                  n_rows, n_cols, nnz, k, stream);
      else if (row_bytes % 128 == 0)
        ok = launch_tma<T, I, 8>(static_cast<const T *>(data), static_cast<const I *>(indices),
                                 static_cast<const I *>(indptr), static_cast<const T *>(rhs), static_cast<T *>(out),
                                 n_rows, n_cols, nnz, k, stream);
    });
  });
  return ok;
}

}  // namespace msx
