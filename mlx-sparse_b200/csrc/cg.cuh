// Conjugate-gradient solvers (plain CG and Jacobi PCG) on the device.
#pragma once
#include "common.cuh"

namespace msx {

constexpr int kStatusRunning = -2147483647 - 1;  // INT_MIN: loop still running

// Device-resident solver state. Scalars never leave the GPU during the solve;
// the host reads `status` once per batch of iterations.
struct CgState {
  double red[4];      // reduction results of the latest reduction kernel
  double rr;          // plain CG: current r.r (double, cg.cpp:123-131)
  double rr_pending;  // plain CG: r.r of the candidate update
  double alpha_d;     // plain CG: step (double)
  double beta_d;      // plain CG: direction update (double)
  float tol;          // max(atol, rtol * ||b||)
  float rho;          // PCG: r.z (float, pcg.cpp:136)
  float alpha_f;      // PCG: step (float)
  float beta_f;       // PCG: direction update (float)
  float true_rr;      // PCG: float(r.r) of the last update
  float residual;     // final residual norm reported to the caller
  int status;         // kStatusRunning, or the final info code
  int completed;      // iterations completed
  int it;             // index of the iteration being run (1-based)
  int maxiter;
  unsigned int counter;  // last-block-done counter of the reductions
  unsigned int round_base;  // peer memory: flag of this solve's halo round 0
  int pad[2];
  double bb_init;     // Chebyshev PCG: b.b and the non-finite count of the
  double bad_init;    // initial residual, kept until r.z is known
  // Timing trace (MSX_CG_TRACE=1, diagnostics only): per reduction kernel
  // (0: SpMV + dots, 1: update) the earliest CTA start of the current
  // launch, and summed over iterations {first CTA start -> last CTA ready,
  // cross-rank all-reduce, count} in globaltimer nanoseconds.
  unsigned long long k_start[2];
  unsigned long long trace[6];
  int tracing;
  int pad2;
};

constexpr int kMaxRanks = 8;  // one node

// Peer-memory mailbox of one rank (IPC-exported), written by the other ranks:
// the fp64 partial sums of the scalar all-reduce in "flagged words" - each
// 64-bit word is (epoch << 32) | one 32-bit half of a double, so a word is
// valid exactly when its flag matches and no fence is needed between data and
// flag. Two slots alternate by epoch parity.
//
// The halo of the search direction travels the same way: each rank owns an
// IPC-exported array of n_halo flagged words (round << 32) | float bits, which
// its peers store into directly and which the SpMV reads (and checks) in place.
struct Mailbox {
  unsigned long long ll[2][kMaxRanks][8];
};

// Counters that persist across solves of one context (never reset, so flags
// in peers' mailboxes stay monotonic).
struct CommState {
  unsigned long long ar_epoch;
  int error;  // 1: a peer wait timed out
};

// What a kernel needs to talk to its peers (passed by value). world == 1
// means no peer-memory exchange (single GPU, or NCCL between kernels).
struct P2pLink {
  Mailbox *mine;
  Mailbox *peer[kMaxRanks];  // every rank's mailbox, mine at [rank]
  CommState *cs;
  const unsigned long long *halo;  // this rank's halo words
  int64_t n_owned;           // halo column j is local column n_owned + j
  int rank, world;
};

// Bytes of one rank's peer-memory descriptor (msx_cg_context_ipc_handles).
constexpr int kCgIpcBytes = 256;

// Multi-GPU layout of one rank (row slab with halo columns; see
// mlx_sparse/distributed.py). Host arrays except send_idx (device).
struct CgDist {
  void *comm;                 // ncclComm_t
  int n_peers;
  const int *peers;           // peer ranks
  const int64_t *send_counts; // per peer: entries of the owned vector sent
  const int64_t *recv_counts; // per peer: halo entries received (halo order)
  const int *send_idx;        // device: concatenated owned indices to send
  int64_t n_halo;
};

struct CgProblem {
  int index_dtype;
  const float *data;
  const void *indices;
  const void *indptr;
  int64_t nnz;
  int64_t n;          // rows owned by this rank (== n_cols on one GPU)
  int64_t n_cols;     // columns of the local matrix (owned + halo)
  const float *b;
  const float *x0;
  const float *inv_diag;  // null for plain CG
  float *x;
  float rtol, atol;
  int maxiter;
  const CgDist *dist = nullptr;  // null: single GPU (NCCL when set)
  // Chebyshev preconditioner (see CgEngineConfig); m_data null: none
  const float *m_data = nullptr;
  const void *m_indices = nullptr;
  const void *m_indptr = nullptr;
  int64_t m_nnz = 0;
  int degree = 0;
  float lambda_min = 0.f, lambda_max = 0.f;
};

struct CgResult {
  int info;
  float residual;
  int iterations;
};

enum CommMode { kCommNone = 0, kCommNccl = 1, kCommP2p = 2 };

// A persistent solver for one matrix (and one rank): plan, buffers and the
// captured iteration graph are built once and reused by every solve.
struct CgEngine;
struct CgEngineConfig {
  int index_dtype;
  const float *data;
  const void *indices;
  const void *indptr;
  int64_t nnz;
  int64_t n;       // owned rows
  int64_t n_halo;  // halo columns
  bool preconditioned;
  int comm;        // CommMode
  int rank, world;
  void *nccl_comm;
  int n_peers;
  const int *peers;
  const int64_t *send_counts;
  const int64_t *recv_counts;
  const int *send_idx;             // device
  const int64_t *peer_dst_offset;  // host, P2P: where this rank's entries land in each peer's p
  // Chebyshev-preconditioned CG (single GPU): the preconditioner matrix M
  // (same index dtype, square, n rows) and the polynomial's degree and
  // spectral interval. m_data == nullptr: no Chebyshev preconditioner.
  const float *m_data = nullptr;
  const void *m_indices = nullptr;
  const void *m_indptr = nullptr;
  int64_t m_nnz = 0;
  int degree = 0;
  float lambda_min = 0.f, lambda_max = 0.f;
};
CgEngine *cg_engine_create(const CgEngineConfig &cfg, cudaStream_t stream);
void cg_engine_destroy(CgEngine *e);
// P2P: kCgIpcBytes per rank: IPC handles of the halo words and the mailbox,
// and the rank's owned length.
void cg_engine_ipc_handles(CgEngine *e, void *out);
void cg_engine_connect(CgEngine *e, const void *all_handles /* world x kCgIpcBytes */);
CgResult cg_engine_solve(CgEngine *e, const float *b, const float *x0, const float *inv_diag, float *x_out,
                         float rtol, float atol, int maxiter, cudaStream_t stream);


// Single-GPU solve on `stream`; synchronises the stream at the end.
CgResult cg_solve(const CgProblem &prob, cudaStream_t stream);

// Chebyshev semi-iteration z = p_d(M) rhs for rhs of n x k (row-major), the
// reference's chebyshev_apply (src/preconditioners/chebyshev/
// chebyshev.cpp:262-300): degree - 1 products with M and fused vector
// updates. Enqueued on `stream`.
void chebyshev_apply_run(int index_dtype, const float *m_data, const void *m_indices, const void *m_indptr,
                         int64_t m_nnz, int64_t n, const float *rhs, int64_t k, float *out, int degree,
                         float lambda_min, float lambda_max, cudaStream_t stream);
// out = inv_diag[row] * rhs (n x k), diagonal_preconditioner_apply.
void diagonal_apply_run(const float *inv_diag, const float *rhs, int64_t n, int64_t k, float *out,
                        cudaStream_t stream);
// Gershgorin bounds and diagonal range {lower, upper, diag_min, diag_max}
// (host); MSX_ERR_INVALID for a non-finite value. Synchronises `stream`.
void gershgorin_run(int index_dtype, const float *data, const void *indices, const void *indptr, int64_t n_rows,
                    float *out4, cudaStream_t stream);

}  // namespace msx
