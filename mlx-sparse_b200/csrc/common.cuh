// Shared helpers for the sm_100a sparse-product kernels: value-type traits
// (fp32 / fp16 / bf16 with fp32 accumulation), error plumbing for the C ABI,
// and stream-ordered scratch allocation.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "msx_sparse.h"

namespace msx {

// ---------------------------------------------------------------------------
// Errors. Host code throws msx::Error; the C-ABI wrapper converts it into a
// status code plus a thread-local message.
// ---------------------------------------------------------------------------
struct Error : public std::runtime_error {
  int status;
  Error(int s, const std::string &m) : std::runtime_error(m), status(s) {}
};

[[noreturn]] inline void fail(int status, const std::string &msg) {
  throw Error(status, msg);
}

#define MSX_CUDA(call)                                                         \
  do {                                                                         \
    cudaError_t err__ = (call);                                                \
    if (err__ != cudaSuccess) {                                                \
      ::msx::fail(MSX_ERR_CUDA, std::string(#call) + " failed: " +             \
                                    cudaGetErrorString(err__));                \
    }                                                                          \
  } while (0)

#define MSX_CHECK_LAUNCH() MSX_CUDA(cudaGetLastError())

// Programmatic dependent launch. A kernel launched with launch(..., pdl=true)
// may be scheduled while the previous kernel in the stream drains; it must call
// pdl_wait() before touching anything that kernel wrote. Kernels call
// pdl_trigger() as soon as they start, so their successor's CTAs fill the SMs
// their own CTAs free. Both are no-ops for ordinary launches.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
void launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
            Args &&...args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = pdl ? attr : nullptr;
  cfg.numAttrs = pdl ? 1 : 0;
  MSX_CUDA(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

void set_last_error(const std::string &msg);

template <typename Fn> int guarded(Fn &&fn) {
  try {
    fn();
    set_last_error("");
    return MSX_OK;
  } catch (const Error &e) {
    set_last_error(e.what());
    return e.status;
  } catch (const std::bad_alloc &) {
    set_last_error("host allocation failed");
    return MSX_ERR_RUNTIME;
  } catch (const std::exception &e) {
    set_last_error(e.what());
    return MSX_ERR_RUNTIME;
  }
}

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

// Keeps memory freed into the current device's default stream-ordered pool
// reserved (release threshold = unlimited) instead of returning it to the
// driver at every synchronisation. Without this, the first scratch allocation
// after a host sync maps fresh memory, which stalls the calling thread for
// milliseconds while the GPU idles. Process-local; done once per device.
inline void keep_pool_memory() {
  static thread_local unsigned long long done = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || (done >> dev & 1ull)) return;
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
    uint64_t threshold = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
  }
  done |= 1ull << dev;
}

// Stream-ordered scratch: freed on the same stream when the guard goes out of
// scope, so the memory is reusable by later work on that stream only.
struct Scratch {
  void *ptr = nullptr;
  cudaStream_t stream = nullptr;
  Scratch(size_t bytes, cudaStream_t s) : stream(s) {
    if (bytes) {
      keep_pool_memory();
      MSX_CUDA(cudaMallocAsync(&ptr, bytes, s));
    }
  }
  ~Scratch() {
    if (ptr) cudaFreeAsync(ptr, stream);
  }
  Scratch(const Scratch &) = delete;
  Scratch &operator=(const Scratch &) = delete;
  template <typename T> T *as() const { return static_cast<T *>(ptr); }
};

inline int num_sms() {
  int dev = 0, sms = 0;
  MSX_CUDA(cudaGetDevice(&dev));
  MSX_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  return sms;
}

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------------------
// Value traits: storage type -> fp32 accumulate, cast back with RNE.
// Mirrors the reference's Accumulator<T> (src/common/common.h:52-79): fp16 and
// bf16 are widened to float before multiplying and the float sum is rounded
// once at the end.
// ---------------------------------------------------------------------------
template <typename T> struct VT;
template <> struct VT<float> {
  __device__ __forceinline__ static float load(float v) { return v; }
  __device__ __forceinline__ static float store(float v) { return v; }
};
template <> struct VT<__half> {
  __device__ __forceinline__ static float load(__half v) { return __half2float(v); }
  __device__ __forceinline__ static __half store(float v) { return __float2half_rn(v); }
};
template <> struct VT<__nv_bfloat16> {
  __device__ __forceinline__ static float load(__nv_bfloat16 v) { return __bfloat162float(v); }
  __device__ __forceinline__ static __nv_bfloat16 store(float v) { return __float2bfloat16_rn(v); }
};

// Multiply/add without FMA contraction so a row summed in one thread reproduces
// the reference's sequential `acc += a * x` rounding exactly.
__device__ __forceinline__ float mul_rn(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float add_rn(float a, float b) { return __fadd_rn(a, b); }

// Streaming (evict-first) loads for matrix arrays read exactly once, so the
// gathered dense operand keeps the L2.
template <typename T> __device__ __forceinline__ T ld_stream(const T *p) { return __ldcs(p); }
template <> __device__ __forceinline__ __half ld_stream<__half>(const __half *p) {
  unsigned short r = __ldcs(reinterpret_cast<const unsigned short *>(p));
  return __ushort_as_half(r);
}
template <> __device__ __forceinline__ __nv_bfloat16 ld_stream<__nv_bfloat16>(const __nv_bfloat16 *p) {
  unsigned short r = __ldcs(reinterpret_cast<const unsigned short *>(p));
  return __ushort_as_bfloat16(r);
}

// Epilogue that only stores y. Epilogues see every finished row (`row`), may
// skip the whole launch (`skip`, evaluated by every thread at entry) and run a
// block-wide `finish` after the CTA's last tile.
struct NoEpilogue {
  static constexpr int kMinBlocks = 8;  // resident CTAs/SM the kernels aim for
  __device__ __forceinline__ bool skip() const { return false; }
  // kHalo: columns >= halo_from() are read through halo_x() (multi-GPU
  // halo words) instead of from x (short-row kernel only).
  static constexpr bool kHalo = false;
  static constexpr bool kShortPipe = false;  // always use the pipelined short-row kernel
  __device__ __forceinline__ int64_t halo_from() const { return INT64_MAX; }
  __device__ __forceinline__ float halo_x(int64_t) { return 0.f; }
  __device__ __forceinline__ void row(int64_t, float) {}
  __device__ __forceinline__ void finish() {}
};

// Dispatch helpers ----------------------------------------------------------
template <typename Fn> void dispatch_value(int vt, Fn &&fn) {
  switch (vt) {
  case MSX_F32: fn(float{}); break;
  case MSX_F16: fn(__half{}); break;
  case MSX_BF16: fn(__nv_bfloat16{}); break;
  default: fail(MSX_ERR_TYPE, "value dtype must be one of float32, float16, bfloat16, got code " + std::to_string(vt) + ".");
  }
}
template <typename Fn> void dispatch_index(int it, Fn &&fn) {
  switch (it) {
  case MSX_I32: fn(int32_t{}); break;
  case MSX_I64: fn(int64_t{}); break;
  default: fail(MSX_ERR_TYPE, "index dtype must be one of int32, int64, got code " + std::to_string(it) + ".");
  }
}

}  // namespace msx
