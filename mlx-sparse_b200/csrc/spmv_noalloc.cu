// msx_csr_matvec_noalloc: the stateless SpMV (merge-path tiles, see spmv.cu)
// with its scratch in a fixed, file-scope device array instead of memory from
// the stream-ordered allocator.
//
// Who needs this: callers that must not allocate device memory at call time -
// for example code running under a custom or pre-reserved memory budget, a
// host framework that forbids allocations inside its execution phase, or an
// application that has already handed all free memory to its own pool. Such
// callers cannot let msx_csr_matvec call cudaMallocAsync for its tile
// partition and split-row partials.
//
// Limits and sharing: the array holds kNoAllocScratchBytes (4 MiB) on every
// GPU that loads the library, for the life of the process. A call needs
// round_up_256(16 + 16 * (n_tiles + 1)) + 8 * n_tiles bytes (tile partition,
// then two float partials per tile), n_tiles = ceil((n_rows + nnz) / 1280),
// i.e. up to about 223 million rows + nonzeros; larger problems are rejected
// with MSX_ERR_INVALID. All calls on a device share the one array, so two calls
// whose kernels overlap on the GPU (different streams, or different host
// threads without ordering) race and corrupt each other's results; order them
// on one stream. The partition is rebuilt on each call, so nothing carried
// over from the previous call is read; the split-row counter is cleared each
// call. Every call looks up the array's device address
// (cudaGetSymbolAddress); the first call on a device may also load the module
// there, so make that first call before any stream capture.
#include "spmv.cuh"

namespace msx {

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the array in the current device's context. The array's
// host-side name is only a stand-in for the symbol, so kernels must be given
// this address. It is looked up on every call (cheap), so it is always the
// address in the context that is current now, also after a device reset.
void *noalloc_scratch_current_device() {
  void *p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || p == nullptr)
    fail(MSX_ERR_CUDA, std::string("cudaGetSymbolAddress for the no-allocation scratch failed: ") +
                           cudaGetErrorString(e));
  return p;
}

}  // namespace

}  // namespace msx

using namespace msx;

extern "C" MSX_API int msx_csr_matvec_noalloc(int value_dtype, int index_dtype, const void *data,
                                              const void *indices, const void *indptr, int64_t nnz, const void *x,
                                              void *y, int64_t n_rows, int64_t n_cols, void *stream) {
  return guarded([&] {
    if (n_rows < 0 || n_cols < 0) fail(MSX_ERR_INVALID, "csr_matvec shape dimensions must be non-negative.");
    if (nnz < 0) fail(MSX_ERR_INVALID, "csr_matvec nnz must be non-negative.");
    dispatch_value(value_dtype, [](auto) {});
    dispatch_index(index_dtype, [](auto) {});
    const int64_t n_tiles = spmv_num_tiles(n_rows, nnz);
    const size_t plan_bytes = spmv_plan_device_bytes(n_tiles);
    const size_t carry_off = (plan_bytes + 255) & ~size_t(255);
    const size_t need = carry_off + sizeof(float) * 2 * (size_t)n_tiles;
    if (need > kNoAllocScratchBytes)
      fail(MSX_ERR_INVALID, "msx_csr_matvec_noalloc: n_rows + nnz = " + std::to_string(n_rows + nnz) +
                                " needs " + std::to_string(need) + " bytes of scratch; the fixed scratch holds " +
                                std::to_string(kNoAllocScratchBytes) + " bytes. Use msx_csr_matvec instead.");
    if ((nnz > 0 && (!data || !indices || !x)) || !indptr || (n_rows > 0 && !y))
      fail(MSX_ERR_INVALID, "csr_matvec arrays must not be null.");
    if (n_rows == 0) return;
    char *base = static_cast<char *>(noalloc_scratch_current_device());
    cudaStream_t s = as_stream(stream);
    spmv_build_plan(index_dtype, indptr, n_rows, nnz, base, n_tiles, s);
    spmv_run(value_dtype, index_dtype, data, indices, indptr, x, y, n_rows, nnz, base, n_tiles, true,
             reinterpret_cast<float *>(base + carry_off), s);
  });
}
