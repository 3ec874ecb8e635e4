/*
 * msx_sparse.h - C ABI of the B200 (sm_100a) sparse-product library.
 *
 * This is the drop-in boundary under the Python `mlx_sparse` package. Each entry
 * point replaces one native op that mlx-sparse's `_native.py` reaches through its
 * nanobind `_ext` module; the reference binding is cited beside each declaration
 * (paths are relative to the mlx-sparse source tree).
 *
 * Conventions
 *  - All array arguments are DEVICE pointers to contiguous (dense, stride-1)
 *    buffers on the current CUDA device. Inputs are borrowed, never consumed.
 *  - `value_dtype` is one of MSX_F32 / MSX_F16 / MSX_BF16; `index_dtype` is
 *    MSX_I32 / MSX_I64 and applies to both `indices` and `indptr`.
 *  - `stream` is a cudaStream_t (NULL = legacy default stream). Work is enqueued
 *    and the call returns without synchronising, except where the reference op
 *    is itself host-synchronising (SpGEMM sizes, solver status).
 *  - Every function returns an msx_status; on failure msx_last_error() returns a
 *    thread-local message. MSX_ERR_INVALID maps to ValueError, MSX_ERR_TYPE to
 *    TypeError, MSX_ERR_OVERFLOW to OverflowError, the rest to RuntimeError.
 *  - Temporary device memory comes from the stream-ordered allocator
 *    (cudaMallocAsync on `stream`), so calls are re-entrant per stream. The
 *    library sets the release threshold of the device's default memory pool
 *    to unlimited (once per device), so freed scratch stays reserved for the
 *    next call instead of being unmapped at every synchronisation.
 */
#ifndef MSX_SPARSE_H
#define MSX_SPARSE_H

#include <stdint.h>

#if defined(__GNUC__)
#define MSX_API __attribute__((visibility("default")))
#else
#define MSX_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum { MSX_F32 = 0, MSX_F16 = 1, MSX_BF16 = 2 } msx_value_dtype;
typedef enum { MSX_I32 = 0, MSX_I64 = 1 } msx_index_dtype;

typedef enum {
  MSX_OK = 0,
  MSX_ERR_INVALID = 1,  /* std::invalid_argument -> ValueError   */
  MSX_ERR_TYPE = 2,     /* dtype problems          -> TypeError    */
  MSX_ERR_OVERFLOW = 3, /* std::overflow_error     -> OverflowError */
  MSX_ERR_RUNTIME = 4,  /* std::runtime_error      -> RuntimeError */
  MSX_ERR_CUDA = 5      /* CUDA runtime failure    -> RuntimeError */
} msx_status;

/* ------------------------------------------------------------------------ */
/* DLPack tensors (the boundary the reference's Python layer crosses with    */
/* device arrays). The layout is the public DLPack ABI (dlpack.h, v0.6-1.x:  */
/* DLTensor has not changed); a caller that already includes dlpack.h gets   */
/* its definitions instead of these.                                         */
/* ------------------------------------------------------------------------ */
#if !defined(DLPACK_VERSION)
typedef struct {
  int32_t device_type; /* kDLCUDA = 2, kDLCUDAManaged = 13 accepted here */
  int32_t device_id;
} DLDevice;
typedef struct {
  uint8_t code; /* kDLInt = 0, kDLFloat = 2, kDLBfloat = 4 */
  uint8_t bits;
  uint16_t lanes;
} DLDataType;
typedef struct {
  void *data;
  DLDevice device;
  int32_t ndim;
  DLDataType dtype;
  int64_t *shape;
  int64_t *strides; /* NULL = compact row-major */
  uint64_t byte_offset;
} DLTensor;
#endif

/* Thread-local message of the last failing call on this thread ("" if none). */
MSX_API const char *msx_last_error(void);

/* Library version and the SM architecture it was compiled for (e.g. 100). */
MSX_API int msx_version(void);
MSX_API int msx_compiled_sm(void);

/* Device-side error check. The SpMV kernels that stage tiles with bulk copies
 * (the tile SpMV when the environment sets MSX_SPMV_TMA=1, read at every
 * call; off by default, plain loads measured faster on B200) wait on
 * shared-memory barriers with a bounded number of polls; if a wait
 * gives up, the kernel stops, records the event in a per-device flag and the
 * rows it had not reached stay unwritten. The flag is sticky: this call
 * synchronises `stream`, reads and clears the flag of the current device and
 * returns MSX_ERR_RUNTIME if it was set. No counterpart in the reference,
 * whose CPU loops cannot time out. */
MSX_API int msx_check_device_errors(void *stream);
/* Test hook: the number of polls those waits make before giving up
 * (default 2^22; 0 makes every wait give up at once; negative restores the
 * default). Process-wide. */
MSX_API int msx_debug_set_spmv_poll_limit(int64_t polls);

/* ------------------------------------------------------------------------ */
/* SpMV plan: row-length bins of a CSR matrix.                              */
/* ------------------------------------------------------------------------ */
/* A plan sorts the row ids once per matrix into bins by row length (1, 2, 4,
 * ... 32 lanes per row, a CTA per row, or 8192-nonzero chunks of one row), so
 * every product runs one balanced launch. It depends only on `indptr`. The
 * reference has no counterpart: its CPU path recomputes nnz-weighted worker
 * ranges on every call (src/common/cpu_parallel.cpp:202-253, reached from
 * src/sparse/csr_matvec/csr_matvec.cpp:156-166).
 * msx_spmv_plan_create allocates device memory (cudaMalloc) and synchronises
 * `stream`; the plan is immutable afterwards and may be shared by concurrent
 * calls on any stream of the same device. */
typedef struct msx_spmv_plan msx_spmv_plan;
MSX_API int msx_spmv_plan_create(int index_dtype, const void *indptr, int64_t n_rows,
                         int64_t nnz, void *stream, msx_spmv_plan **out);
MSX_API int msx_spmv_plan_destroy(msx_spmv_plan *plan);
/* Blocks of one product launch, and rows split into several chunks. */
MSX_API int msx_spmv_plan_info(const msx_spmv_plan *plan, int64_t *n_blocks,
                       int64_t *n_long_rows);

/* y = A @ x. Replaces `csr_matvec(data, indices, indptr, x, n_rows, n_cols)`
 * (src/bindings.cpp:874-883 -> src/sparse/csr_matvec/csr_matvec.cpp:326-356,
 * CPU loop :79-168). With a plan the binned kernel runs; `plan` may be NULL,
 * in which case an nnz-balanced merge-path partition is built in stream-ordered
 * scratch on every call. A plan must have been created for this matrix's
 * indptr, n_rows and nnz. fp16/bf16 accumulate in fp32. */
MSX_API int msx_csr_matvec(int value_dtype, int index_dtype, const void *data,
                   const void *indices, const void *indptr, int64_t nnz,
                   const void *x, void *y, int64_t n_rows, int64_t n_cols,
                   const msx_spmv_plan *plan, void *stream);

/* y = A @ x without allocating any device memory. No counterpart in the
 * reference: it exists for callers that cannot allocate at call time (a
 * pre-reserved memory budget, an execution phase where allocation is
 * forbidden, or all free memory already handed to the caller's own pool).
 * Same algorithm and results as msx_csr_matvec with plan == NULL, but the
 * tile partition and split-row partials live in one fixed 4 MiB device array
 * per GPU (held from library load until exit), which limits n_rows + nnz to
 * about 223 million; larger inputs return MSX_ERR_INVALID. Every call looks
 * up that array's device address (cudaGetSymbolAddress); the first call on a
 * device may also load the module there, so make it before any stream
 * capture. All calls share the array: calls whose work
 * overlaps on the GPU race and must be ordered on one stream. */
MSX_API int msx_csr_matvec_noalloc(int value_dtype, int index_dtype,
                                   const void *data, const void *indices,
                                   const void *indptr, int64_t nnz,
                                   const void *x, void *y, int64_t n_rows,
                                   int64_t n_cols, void *stream);

/* Y = A @ B for a row-major dense B[n_cols, k] -> Y[n_rows, k]. Replaces
 * `csr_matmul(data, indices, indptr, rhs, n_rows, n_cols)`
 * (src/bindings.cpp:965-975 -> src/sparse/csr_matmul/csr_matmul.cpp:383-418,
 * CPU loop :83-222). fp16/bf16 accumulate in fp32. */
MSX_API int msx_csr_matmul(int value_dtype, int index_dtype, const void *data,
                   const void *indices, const void *indptr, int64_t nnz,
                   const void *rhs, int64_t rhs_cols, void *out, int64_t n_rows,
                   int64_t n_cols, void *stream);

/* ------------------------------------------------------------------------ */
/* COO entry, transposition and the backward products.                      */
/* ------------------------------------------------------------------------ */
/* COO -> CSR. Replaces `coo_tocsr(data, row, col, n_rows, n_cols)`
 * (src/bindings.cpp -> src/sparse/coo_tocsr/coo_tocsr.cpp:94-237,
 * mlx_sparse/_coo.py:126-154). `row`/`col` share `index_dtype`; the outputs
 * (caller-allocated) are out_data[nnz] (may be NULL: structure only),
 * out_indices[nnz] (col's dtype), out_indptr[n_rows + 1] (row's dtype) and,
 * optionally, out_perm[nnz] (int64: source position of every output entry,
 * which is what the reference's coo_tocsr data VJP gathers through,
 * coo_tocsr.cpp:237-300). sort_columns = 1 orders each row by column, then
 * source position (the reference's coo_tocsr, duplicates kept); 0 keeps each
 * row in source order (the summation order of the reference's coo_matmul,
 * src/sparse/coo_matmul/coo_matmul.cpp). Coordinates outside the shape
 * return MSX_ERR_INVALID. Synchronises `stream` once. */
MSX_API int msx_coo_tocsr(int value_dtype, int index_dtype, const void *data,
                          const void *row, const void *col, int64_t nnz,
                          int64_t n_rows, int64_t n_cols, int sort_columns,
                          void *out_data, void *out_indices, void *out_indptr,
                          int64_t *out_perm, void *stream);

/* CSR of A^T (n_cols x n_rows): row c lists column c's entries of A by
 * ascending row (so the result has sorted indices). Replaces
 * `csr_transpose` (src/sparse/csr_transpose). out_perm as msx_coo_tocsr.
 * Synchronises `stream` once. */
MSX_API int msx_csr_transpose(int value_dtype, int index_dtype, const void *data,
                              const void *indices, const void *indptr,
                              int64_t nnz, int64_t n_rows, int64_t n_cols,
                              void *out_data, void *out_indices,
                              void *out_indptr, int64_t *out_perm,
                              void *stream);

/* out = A^T @ x (x[n_rows] -> out[n_cols]) and out = A^T @ B
 * (B[n_rows, rhs_cols] -> out[n_cols, rhs_cols]). Replace
 * `csr_matvec_transpose` (src/sparse/csr_matvec_transpose/
 * csr_matvec_transpose.cpp:76-97, the VJP of csr_matvec with respect to x,
 * src/sparse/csr_matvec/csr_matvec.cpp:247-257) and `csr_matmul_transpose`
 * (src/sparse/csr_matmul_transpose). Every output element sums its column's
 * entries in row-major order, as the reference's serial loop does. The
 * transposed structure is built in stream scratch on every call (the Python
 * layer caches it per matrix and calls the plain products instead);
 * synchronises `stream` once. */
MSX_API int msx_csr_matvec_transpose(int value_dtype, int index_dtype,
                                     const void *data, const void *indices,
                                     const void *indptr, int64_t nnz,
                                     const void *x, void *out, int64_t n_rows,
                                     int64_t n_cols, void *stream);
MSX_API int msx_csr_matmul_transpose(int value_dtype, int index_dtype,
                                     const void *data, const void *indices,
                                     const void *indptr, int64_t nnz,
                                     const void *rhs, int64_t rhs_cols,
                                     void *out, int64_t n_rows, int64_t n_cols,
                                     void *stream);

/* Cotangent of the stored values. matvec: out[p] = cot[row(p)] * x[col(p)];
 * matmul: out[p] = sum_j cot[row(p), j] * B[col(p), j], j in order, fp32
 * accumulation. Replace `csr_matvec_data_vjp` (src/sparse/
 * csr_matvec_data_vjp) and `csr_matmul_data_vjp` (src/sparse/
 * csr_matmul_data_vjp/csr_matmul_data_vjp.cpp:88-100). */
MSX_API int msx_csr_matvec_data_vjp(int value_dtype, int index_dtype,
                                    const void *indices, const void *indptr,
                                    int64_t nnz, const void *x,
                                    const void *cotangent, void *out,
                                    int64_t n_rows, int64_t n_cols,
                                    void *stream);
MSX_API int msx_csr_matmul_data_vjp(int value_dtype, int index_dtype,
                                    const void *indices, const void *indptr,
                                    int64_t nnz, const void *rhs,
                                    const void *cotangent, int64_t rhs_cols,
                                    void *out, int64_t n_rows, int64_t n_cols,
                                    void *stream);

/* ------------------------------------------------------------------------ */
/* SpGEMM C = A @ B, canonical (sorted, duplicate-free, exact zeros pruned). */
/* ------------------------------------------------------------------------ */
/* Batched products with one matrix, replacing csr_batched_matvec
 * (src/bindings.cpp:907-915; src/sparse/csr_batched_matvec/
 * csr_batched_matvec.cpp:82-130) and csr_batched_matmul (src/bindings.cpp:
 * 1000-1008). rhs is [batch, n_cols] (matvec) or [batch, n_cols, rhs_cols]
 * (matmul), row-major and contiguous; out is [batch, n_rows] or
 * [batch, n_rows, rhs_cols]. Every output element sums its row's nonzeros in
 * order, as the reference does. */
MSX_API int msx_csr_batched_matvec(int value_dtype, int index_dtype,
                                   const void *data, const void *indices,
                                   const void *indptr, int64_t nnz,
                                   const void *rhs, int64_t batch, void *out,
                                   int64_t n_rows, int64_t n_cols, void *stream);
MSX_API int msx_csr_batched_matmul(int value_dtype, int index_dtype,
                                   const void *data, const void *indices,
                                   const void *indptr, int64_t nnz,
                                   const void *rhs, int64_t batch,
                                   int64_t rhs_cols, void *out, int64_t n_rows,
                                   int64_t n_cols, void *stream);

/* Replaces `csr_matmat(lhs_data, lhs_indices, lhs_indptr, rhs_data,
 * rhs_indices, rhs_indptr, lhs_n_rows, lhs_n_cols, rhs_n_rows, rhs_n_cols)`
 * (src/bindings.cpp:1116-1131 -> src/sparse/csr_matmat/csr_matmat.cpp:1319-1424,
 * host Gustavson :544-817). Two-call protocol because the output size is data
 * dependent:
 *   1. msx_csr_matmat_symbolic computes the exact output row counts (after
 *      zero pruning), writes the output indptr[lhs_n_rows + 1] (dtype
 *      `out_index_dtype`) and returns the total in *out_nnz (synchronises
 *      `stream`, as the reference's host path does).
 *   2. msx_csr_matmat_numeric fills caller-allocated out_data[out_nnz] and
 *      out_indices[out_nnz] using that indptr.
 * The output index dtype follows the reference rule (:1354-1356): the inputs'
 * dtype when lhs and rhs agree, else int64. Each output value is accumulated
 * in the reference's order (lhs position, then rhs position) in fp32, so
 * exact cancellations agree. `prune_zeros` = 1 drops entries whose stored
 * value is exactly zero (the reference's csr_matmat behaviour, :613-641);
 * 0 keeps them (used for duplicate summation, I @ A). */
MSX_API int msx_csr_matmat_symbolic(int value_dtype, int lhs_index_dtype,
                            const void *lhs_data, const void *lhs_indices,
                            const void *lhs_indptr, int64_t lhs_nnz,
                            int rhs_index_dtype, const void *rhs_data,
                            const void *rhs_indices, const void *rhs_indptr,
                            int64_t rhs_nnz, int64_t lhs_n_rows,
                            int64_t lhs_n_cols, int64_t rhs_n_rows,
                            int64_t rhs_n_cols, int out_index_dtype,
                            void *out_indptr, int64_t *out_nnz,
                            int prune_zeros, void *stream);
MSX_API int msx_csr_matmat_numeric(int value_dtype, int lhs_index_dtype,
                           const void *lhs_data, const void *lhs_indices,
                           const void *lhs_indptr, int64_t lhs_nnz,
                           int rhs_index_dtype, const void *rhs_data,
                           const void *rhs_indices, const void *rhs_indptr,
                           int64_t rhs_nnz, int64_t lhs_n_rows,
                           int64_t lhs_n_cols, int64_t rhs_n_rows,
                           int64_t rhs_n_cols, int out_index_dtype,
                           const void *out_indptr, int64_t out_nnz,
                           void *out_data, void *out_indices,
                           int prune_zeros, void *stream);

/* ------------------------------------------------------------------------ */
/* Conjugate gradients (fp32 values, int32/int64 indices).                   */
/* ------------------------------------------------------------------------ */
/* Plain CG. Replaces `csr_cg(data, indices, indptr, b, x0, n_rows, n_cols,
 * rtol, atol, maxiter)` (src/bindings.cpp:1133-1145 -> src/linalg/cg/cg.cpp:
 * 338-379, CPU loop :75-256). Writes x_out[n_rows] on the device and the
 * scalars *info (0 converged, >0 iteration budget exhausted, -1 breakdown,
 * -3 non-finite), *residual and *iterations on the HOST (the call synchronises
 * `stream` at the end, like the reference's finish_solver_result). */
MSX_API int msx_csr_cg(int index_dtype, const float *data, const void *indices,
               const void *indptr, int64_t nnz, const float *b,
               const float *x0, float *x_out, int64_t n_rows, int64_t n_cols,
               float rtol, float atol, int32_t maxiter, int32_t *info,
               float *residual, int32_t *iterations, void *stream);

/* Jacobi-preconditioned CG. Replaces `csr_pcg_jacobi(data, indices, indptr, b,
 * x0, inv_diag, n_rows, n_cols, rtol, atol, maxiter)` (src/bindings.cpp:
 * 1147-1161 -> src/preconditioners/pcg/pcg.cpp:317-366, CPU loop :70-230).
 * Status -2 = non-positive preconditioned inner product. */
MSX_API int msx_csr_pcg_jacobi(int index_dtype, const float *data, const void *indices,
                       const void *indptr, int64_t nnz, const float *b,
                       const float *x0, const float *inv_diag, float *x_out,
                       int64_t n_rows, int64_t n_cols, float rtol, float atol,
                       int32_t maxiter, int32_t *info, float *residual,
                       int32_t *iterations, void *stream);

/* Chebyshev-preconditioned CG. Replaces `csr_pcg_chebyshev(data, indices,
 * indptr, b, x0, m_data, m_indices, m_indptr, n_rows, n_cols, degree,
 * lambda_min, lambda_max, rtol, atol, maxiter)` (mlx_sparse/_native.py:
 * 1211-1260 -> src/preconditioners/pcg/chebyshev.cpp:124-313): Jacobi-PCG's
 * recurrence and statuses with z = p_d(M) r, the first-kind Chebyshev
 * semi-iteration of `degree` terms on the preconditioner matrix M
 * (m_*, square n_rows, same index dtype) over [lambda_min, lambda_max].
 * Single GPU; synchronises `stream` at the end. */
MSX_API int msx_csr_pcg_chebyshev(int index_dtype, const float *data,
                                  const void *indices, const void *indptr,
                                  int64_t nnz, const float *b, const float *x0,
                                  const float *m_data, const void *m_indices,
                                  const void *m_indptr, int64_t m_nnz,
                                  float *x_out, int64_t n_rows, int64_t n_cols,
                                  int32_t degree, float lambda_min,
                                  float lambda_max, float rtol, float atol,
                                  int32_t maxiter, int32_t *info,
                                  float *residual, int32_t *iterations,
                                  void *stream);

/* out = p_d(M) rhs for rhs of n x rhs_cols (row-major; 1 column = a vector).
 * Replaces `csr_chebyshev_preconditioner_apply` (src/preconditioners/
 * chebyshev/chebyshev.cpp:262-300). */
MSX_API int msx_csr_chebyshev_apply(int index_dtype, const float *m_data,
                                    const void *m_indices, const void *m_indptr,
                                    int64_t m_nnz, int64_t n, const float *rhs,
                                    int64_t rhs_cols, float *out,
                                    int32_t degree, float lambda_min,
                                    float lambda_max, void *stream);

/* out[row, c] = inv_diag[row] * rhs[row, c]. Replaces
 * `diagonal_preconditioner_apply` (src/preconditioners/diagonal/
 * diagonal.cpp:60-88, 120-161). */
MSX_API int msx_diagonal_preconditioner_apply(const float *inv_diag,
                                              const float *rhs, int64_t n,
                                              int64_t rhs_cols, float *out,
                                              void *stream);

/* Gershgorin bounds and the diagonal range of a square fp32 CSR matrix into
 * host out4 = {lower, upper, diag_min, diag_max}: the Gershgorin part of
 * `csr_chebyshev_spectral_bounds` (src/preconditioners/chebyshev/
 * chebyshev.cpp:120-161). Non-finite values return MSX_ERR_INVALID.
 * Synchronises `stream`. */
MSX_API int msx_csr_gershgorin_bounds(int index_dtype, const float *data,
                                      const void *indices, const void *indptr,
                                      int64_t nnz, int64_t n_rows,
                                      int64_t n_cols, float *out4,
                                      void *stream);

/* Main diagonal of a CSR matrix into out[min(n_rows, n_cols)], duplicate
 * entries summed in stored order (fp32 accumulation). Replaces the native
 * `csr_diagonal` that mlx-sparse's preconditioners.jacobi() calls
 * (mlx_sparse/linalg/preconditioners.py:1108 -> src/sparse/csr_diagonal). */
MSX_API int msx_csr_diagonal(int value_dtype, int index_dtype, const void *data,
                             const void *indices, const void *indptr,
                             int64_t nnz, int64_t n_rows, int64_t n_cols,
                             void *out, void *stream);

/* ------------------------------------------------------------------------ */
/* Multi-GPU CG over row slabs (one process per GPU, NCCL over NVLink).      */
/* ------------------------------------------------------------------------ */
/* No counterpart in the reference, which runs on one device only (its CPU
 * threads split rows by nnz-weighted ranges, src/common/cpu_parallel.cpp:
 * 202-253; the same partition is applied here to GPUs). A communicator is
 * created collectively: rank 0 calls msx_dist_unique_id, the 128-byte id is
 * broadcast by the caller, every rank calls msx_dist_comm_create on its
 * current device. */
MSX_API int msx_dist_unique_id(void *out, int64_t size);
MSX_API int msx_dist_comm_create(const void *unique_id, int nranks, int rank,
                                 void **comm);
MSX_API int msx_dist_comm_destroy(void *comm);

/* CG (inv_diag == NULL) or Jacobi PCG of the global system, called by every
 * rank with its slab: rows [r0, r0 + n_owned) of A with local column ids
 * (owned columns first, then n_halo halo columns in owner order), its owned
 * entries of b, x0 and inv_diag, and the halo lists: for each of n_peers
 * peers (host arrays) the number of owned entries it needs (send_counts, the
 * owned indices concatenated in device array send_idx) and the number of halo
 * entries received from it (recv_counts). Same recurrence, statuses and
 * residual as msx_csr_cg / msx_csr_pcg_jacobi (src/linalg/cg/cg.cpp:75-256,
 * src/preconditioners/pcg/pcg.cpp:70-230); the scalars returned are
 * identical on every rank. */
MSX_API int msx_dist_pcg(void *comm, int index_dtype, const float *data,
                         const void *indices, const void *indptr, int64_t nnz,
                         int64_t n_owned, int64_t n_halo, const float *b,
                         const float *x0, const float *inv_diag, float *x_out,
                         float rtol, float atol, int32_t maxiter, int n_peers,
                         const int *peers, const int64_t *send_counts,
                         const int64_t *recv_counts, const int *send_idx,
                         int32_t *info, float *residual, int32_t *iterations,
                         void *stream);

/* Persistent CG solver for one matrix (and one rank): the row bins, work
 * buffers and the CUDA graph of a batch of iterations are built once and reused
 * by every msx_cg_context_solve, so repeated solves skip all setup. No
 * counterpart in the reference (its csr_cg / csr_pcg_jacobi primitives,
 * src/linalg/cg/cg.cpp:338-379, src/preconditioners/pcg/pcg.cpp:317-366,
 * rebuild everything per call); the solve itself is the same recurrence.
 * comm_mode: 0 single GPU, 1 NCCL (nccl_comm from msx_dist_comm_create),
 * 2 peer memory over NVLink: every rank exports a descriptor of
 * MSX_CG_IPC_BYTES (IPC handles of its two direction buffers and its mailbox,
 * msx_cg_context_ipc_handles), the caller gathers them in rank order and
 * passes all of them to msx_cg_context_connect before the first solve;
 * peer_dst_offset[k] is where this rank's entries for peer k start in that
 * peer's p vector (its owned length plus the offset of this rank's block in
 * its halo). All ranks must call solve together; peer waits are bounded and a
 * lost peer ends the solve with an error instead of hanging. */
typedef struct msx_cg_context msx_cg_context;
#define MSX_CG_IPC_BYTES 256
MSX_API int msx_cg_context_create(int index_dtype, const float *data,
                                  const void *indices, const void *indptr,
                                  int64_t nnz, int64_t n_owned, int64_t n_halo,
                                  int preconditioned, int comm_mode, int rank,
                                  int world, void *nccl_comm, int n_peers,
                                  const int *peers, const int64_t *send_counts,
                                  const int64_t *recv_counts, const int *send_idx,
                                  const int64_t *peer_dst_offset, void *stream,
                                  msx_cg_context **out);
MSX_API int msx_cg_context_ipc_handles(msx_cg_context *ctx, void *out,
                                       int64_t size);
MSX_API int msx_cg_context_connect(msx_cg_context *ctx, const void *all_handles,
                                   int64_t size);
MSX_API int msx_cg_context_solve(msx_cg_context *ctx, const float *b,
                                 const float *x0, const float *inv_diag,
                                 float *x_out, float rtol, float atol,
                                 int32_t maxiter, int32_t *info, float *residual,
                                 int32_t *iterations, void *stream);
MSX_API int msx_cg_context_destroy(msx_cg_context *ctx);

/* ------------------------------------------------------------------------ */
/* DLPack entry points: the same operations with every array passed as a     */
/* DLTensor (borrowed; outputs caller-allocated). They check what the raw    */
/* entry points cannot: device (CUDA, the current device), dtype codes,      */
/* ranks, shapes against n_rows / n_cols, compact strides, and that indices  */
/* and indptr share an index dtype; byte_offset is honoured. Errors follow    */
/* the same status codes and messages as the reference's front-ends.         */
/* ------------------------------------------------------------------------ */
/* csr_matvec (src/bindings.cpp:874-883, mlx_sparse/_native.py:179-189). */
MSX_API int msx_dl_csr_matvec(const DLTensor *data, const DLTensor *indices,
                              const DLTensor *indptr, const DLTensor *x,
                              DLTensor *y, int64_t n_rows, int64_t n_cols,
                              const msx_spmv_plan *plan, void *stream);
/* csr_matmul (src/bindings.cpp:965-975, mlx_sparse/_native.py:286-296). */
MSX_API int msx_dl_csr_matmul(const DLTensor *data, const DLTensor *indices,
                              const DLTensor *indptr, const DLTensor *rhs,
                              DLTensor *out, int64_t n_rows, int64_t n_cols,
                              void *stream);
/* csr_matmat, two calls (src/bindings.cpp:1116-1131,
 * mlx_sparse/_native.py:393-408): the symbolic call fills out_indptr
 * (int32 when both operands are int32, else int64) and *out_nnz; the numeric
 * call fills out_data and out_indices (same index dtype as out_indptr). */
MSX_API int msx_dl_csr_matmat_symbolic(
    const DLTensor *lhs_data, const DLTensor *lhs_indices,
    const DLTensor *lhs_indptr, const DLTensor *rhs_data,
    const DLTensor *rhs_indices, const DLTensor *rhs_indptr, int64_t lhs_n_rows,
    int64_t lhs_n_cols, int64_t rhs_n_rows, int64_t rhs_n_cols,
    DLTensor *out_indptr, int64_t *out_nnz, int prune_zeros, void *stream);
MSX_API int msx_dl_csr_matmat_numeric(
    const DLTensor *lhs_data, const DLTensor *lhs_indices,
    const DLTensor *lhs_indptr, const DLTensor *rhs_data,
    const DLTensor *rhs_indices, const DLTensor *rhs_indptr, int64_t lhs_n_rows,
    int64_t lhs_n_cols, int64_t rhs_n_rows, int64_t rhs_n_cols,
    const DLTensor *out_indptr, DLTensor *out_data, DLTensor *out_indices,
    int prune_zeros, void *stream);
/* csr_cg / csr_pcg_jacobi (src/bindings.cpp:1133-1161,
 * mlx_sparse/_native.py:883-909, 1139-1167); scalars as msx_csr_cg. */
MSX_API int msx_dl_csr_cg(const DLTensor *data, const DLTensor *indices,
                          const DLTensor *indptr, const DLTensor *b,
                          const DLTensor *x0, DLTensor *x_out, int64_t n_rows,
                          int64_t n_cols, float rtol, float atol,
                          int32_t maxiter, int32_t *info, float *residual,
                          int32_t *iterations, void *stream);
MSX_API int msx_dl_csr_pcg_jacobi(const DLTensor *data, const DLTensor *indices,
                                  const DLTensor *indptr, const DLTensor *b,
                                  const DLTensor *x0, const DLTensor *inv_diag,
                                  DLTensor *x_out, int64_t n_rows,
                                  int64_t n_cols, float rtol, float atol,
                                  int32_t maxiter, int32_t *info,
                                  float *residual, int32_t *iterations,
                                  void *stream);

#ifdef __cplusplus
}
#endif

#endif /* MSX_SPARSE_H */
