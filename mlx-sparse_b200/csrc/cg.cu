// Plain CG and Jacobi-preconditioned CG with the whole Krylov loop on the
// device, on one GPU or as one rank of a row-sharded solve.
//
// Reference behaviour (restated step by step, same scalar types):
//   plain CG   src/linalg/cg/cg.cpp:75-256 - double dots, x/r/p updated in
//              double and stored as float, element-wise non-finite skip,
//              scaled breakdown test only when |p.Ap| <= eps.
//   Jacobi PCG src/preconditioners/pcg/pcg.cpp:70-230 - float scalars from
//              double-accumulated dots (dot_float, linalg/common/common.h:47-59),
//              float vector updates, statuses 0 / maxiter / -1 / -2 / -3.
//
// B200 design: one iteration is three kernels:
//   K1  SpMV p -> Ap with the row-length-binned kernel (spmv_binned.cuh) and
//       p.Ap, p.p, Ap.Ap fused into its row epilogue (every row is written
//       once, final);
//   K2  the x/r(/z) update with r.r (and r.z) fused;
//   K3  the direction update p = r + beta p (or z + beta p).
// Each reduction writes one fp64 partial per CTA; the last CTA to finish
// (atomic ticket) sums the partials in CTA order - deterministic - and makes
// the reference's scalar decisions in one thread, writing alpha/beta/status to
// a device state block. Later kernels read the state and return at once when
// the solve has stopped, so batches of iterations are captured in a CUDA graph
// and launched back to back; the host reads the status once per batch.
// Matrices with rows longer than the CTA bin (split into chunks) run the plain
// SpMV + chunk fixup and a separate dot kernel instead of the fused K1.
//
// Row-sharded (one rank per GPU of a node), peer-memory mode: K3's first CTAs
// store the direction entries the peers read straight into the peers' halo
// word arrays; K1 reads halo columns from this rank's word array, checking
// each word's round flag; the last CTA of each reduction exchanges flagged
// fp64 partial-sum words through the ranks' mailboxes and adds them in rank
// order before deciding. Still three kernels per iteration. NCCL mode adds a
// send/recv of the halo before K1 and an all-reduce + decision kernel after
// each reduction. The solver state (plan, buffers, captured graph) lives in a
// CgEngine that is reused across solves.
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>
#if defined(MSX_HAVE_NCCL)
#include <nccl.h>
#endif

#include "cg.cuh"
#include "spmv.cuh"
#include "spmv_binned.cuh"
#include <memory>

namespace msx {

namespace {

constexpr int kThreads = 256;

enum Kind { kCG = 0, kPCG = 1, kCheb = 2 };

__device__ __forceinline__ bool finite_f(float v) { return isfinite(v); }
__device__ __forceinline__ bool finite_d(double v) { return isfinite(v); }
__device__ __forceinline__ bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Block-wide sum of 4 doubles; the result is valid in thread 0.
__device__ __forceinline__ void block_sum4(double (&v)[4], double *smem /*[32*4]*/) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v[c] += __shfl_down_sync(0xffffffffu, v[c], off);
  if (lane == 0)
#pragma unroll
    for (int c = 0; c < 4; ++c) smem[warp * 4 + c] = v[c];
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      double s = lane < nw ? smem[lane * 4 + c] : 0.0;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_down_sync(0xffffffffu, s, off);
      v[c] = s;
    }
  }
  __syncthreads();
}

// Writes this CTA's partial and, in the last CTA to finish, the ordered sum of
// all partials into state->red. Returns true in every thread of the last CTA.
__device__ bool reduce_last(double (&v)[4], double *partials, CgState *st) {
  __shared__ double smem[32 * 4];
  __shared__ bool is_last;
  block_sum4(v, smem);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int c = 0; c < 4; ++c) partials[blockIdx.x * 4 + c] = v[c];
    __threadfence();
    const unsigned ticket = atomicAdd(&st->counter, 1u);
    is_last = (ticket == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return false;
  __threadfence();
  double s[4] = {0.0, 0.0, 0.0, 0.0};
  for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x)
#pragma unroll
    for (int c = 0; c < 4; ++c) s[c] += __ldcg(partials + b * 4 + c);
  block_sum4(s, smem);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int c = 0; c < 4; ++c) st->red[c] = s[c];
    st->counter = 0;
  }
  __syncthreads();
  return true;
}

// ---- peer memory (one node, NVLink) ------------------------------------------------
constexpr long long kPeerPollLimit = 1ll << 24;

__device__ __forceinline__ void st_relaxed_sys(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Sums st->red (4 doubles) over the ranks through their mailboxes. Run by one
// full warp. Every rank stores its 8 flagged words into every mailbox (its own
// included), then waits, bounded, for the words of all ranks and adds them in
// rank order, so every rank computes identical scalars. Returns false on a
// timeout.
__device__ bool ll_allreduce(CgState *st, const P2pLink *L) {
  __shared__ unsigned halves[kMaxRanks][8];
  const int lane = threadIdx.x & 31;
  unsigned epoch = 0;
  if (lane == 0) {
    epoch = (unsigned)(L->cs->ar_epoch + 1);
    L->cs->ar_epoch = epoch;
  }
  epoch = __shfl_sync(0xffffffffu, epoch, 0);
  const int slot = (int)(epoch & 1u);
  const int word = lane & 7;
  const unsigned long long bits = (unsigned long long)__double_as_longlong(st->red[word >> 1]);
  const unsigned half = (word & 1) ? (unsigned)(bits >> 32) : (unsigned)bits;
  const unsigned long long w = ((unsigned long long)epoch << 32) | half;
  const int total = 8 * L->world;
  for (int i = lane; i < total; i += 32) st_relaxed_sys(&L->peer[i >> 3]->ll[slot][L->rank][word], w);
  bool ok = true;
  for (int i = lane; i < total; i += 32) {
    const unsigned long long *src = &L->mine->ll[slot][i >> 3][word];
    unsigned long long v = ld_relaxed_sys(src);
    long long polls = 0;
    while ((unsigned)(v >> 32) != epoch) {
      if (++polls > kPeerPollLimit) {
        ok = false;
        break;
      }
      v = ld_relaxed_sys(src);
    }
    halves[i >> 3][word] = (unsigned)v;
  }
  ok = __all_sync(0xffffffffu, ok);
  __syncwarp();
  if (ok && lane < 4) {
    double sum = 0.0;
    for (int q = 0; q < L->world; ++q) {
      const unsigned long long b = ((unsigned long long)halves[q][2 * lane + 1] << 32) | halves[q][2 * lane];
      sum += __longlong_as_double((long long)b);
    }
    st->red[lane] = sum;
  }
  __syncwarp();
  return ok;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Trace hook at a reduction kernel's start (slot 0: SpMV + dots, 1: update).
__device__ __forceinline__ void trace_start(CgState *st, int slot) {
  if (st->tracing && threadIdx.x == 0) atomicMin(&st->k_start[slot], global_ns());
}

// The last CTA of a reduction: combine over the ranks (peer memory) and run
// the decision `f` in one thread. Single GPU: decide directly when `decide`.
template <typename F>
__device__ __forceinline__ void reduce_and_decide(double (&v)[4], double *partials, CgState *st, const P2pLink *L,
                                                  bool decide, F f, int trace_slot = -1) {
  if (!reduce_last(v, partials, st)) return;
  unsigned long long t_ready = 0;
  if (threadIdx.x == 0 && trace_slot >= 0 && st->tracing) t_ready = global_ns();
  auto trace_done = [&]() {
    if (trace_slot >= 0 && st->tracing) {
      const unsigned long long t_done = global_ns();
      st->trace[3 * trace_slot] += t_ready - st->k_start[trace_slot];
      st->trace[3 * trace_slot + 1] += t_done - t_ready;
      st->trace[3 * trace_slot + 2] += 1;
      st->k_start[trace_slot] = ~0ull;
    }
  };
  if (L) {
    if (threadIdx.x < 32) {
      const bool ok = ll_allreduce(st, L);
      if (threadIdx.x == 0) {
        trace_done();
        if (ok) {
          f();
        } else {
          L->cs->error = 1;
          st->status = -4;  // communication timeout (not a reference status)
        }
      }
    }
  } else if (threadIdx.x == 0 && decide) {
    trace_done();
    f();
  }
}

// ---- halo words ----------------------------------------------------------------
// Halo column j of the current search direction is the word halo[j] of round r
// when its flag equals r. Rounds are numbered per solve from
// st->round_base: 0 for x0, then st->it for the direction iteration `it`
// reads. A producer only writes round r + 1 after every rank has finished
// reading round r (the scalar all-reduces in between order them), so one
// array per rank suffices.
__device__ __forceinline__ unsigned long long halo_word(unsigned round, float v) {
  return ((unsigned long long)round << 32) | __float_as_uint(v);
}

// Reads halo column j of `round`, waiting (bounded) for the owner's store.
// On a timeout it marks the solve failed and returns 0.
__device__ __noinline__ float halo_wait_read(CgState *st, const P2pLink *L, int64_t j, unsigned round) {
  const unsigned long long *w = L->halo + j;
  long long polls = 0;
  while (true) {
    const unsigned long long v = ld_relaxed_sys(w);
    if ((unsigned)(v >> 32) == round) return __uint_as_float((unsigned)v);
    if (++polls > kPeerPollLimit || ((polls & 255) == 0 && *(volatile int *)&L->cs->error)) {
      L->cs->error = 1;
      st->status = -4;
      return 0.f;
    }
  }
}

__device__ __forceinline__ float halo_read(CgState *st, const P2pLink *L, int64_t j, unsigned round) {
  const unsigned long long v = ld_relaxed_sys(L->halo + j);
  if ((unsigned)(v >> 32) == round) return __uint_as_float((unsigned)v);
  return halo_wait_read(st, L, j, round);
}

// Where one rank's halo entries go: for each receiving peer, its halo words
// where this rank's block starts, and the prefix of the send counts over the
// concatenated send list `idx`. The first `ctas` CTAs of a kernel push.
struct PushPlan {
  unsigned long long *dst[kMaxRanks];
  long long off[kMaxRanks + 1];
  int n_peers;
  int ctas;
  const int *idx;
};

__device__ __forceinline__ int push_ctas(const PushPlan *pp) { return min((int)gridDim.x, pp->ctas); }

// Stores value(i) of round `round` for every send entry i into the peers'
// halo words (pushing CTAs only). No fence: each word carries its own flag.
template <typename F> __device__ __forceinline__ void halo_push(const PushPlan *pp, unsigned round, F value) {
  const int P = push_ctas(pp);
  if ((int)blockIdx.x >= P) return;
  const long long ns = pp->off[pp->n_peers];
  for (long long j = blockIdx.x * (long long)blockDim.x + threadIdx.x; j < ns; j += (long long)P * blockDim.x) {
    int k = 0;
    while (k + 1 < pp->n_peers && j >= pp->off[k + 1]) ++k;
    st_relaxed_sys(pp->dst[k] + (j - pp->off[k]), halo_word(round, value(pp->idx[j])));
  }
}

// ---- scalar decisions (one thread) -------------------------------------------
// After the initial residual: red = {b.b, r.r, r.z, nonfinite}.
__device__ void decide_init(CgState *st, int kind, float rtol, float atol) {
  const double bb = st->red[0], rr = st->red[1], rz = st->red[2];
  const bool finite = st->red[3] == 0.0;
  const float b_norm = (float)sqrt(fmax(bb, 0.0));
  const float tol = fmaxf(atol, __fmul_rn(rtol, b_norm));
  st->tol = tol;
  st->completed = 0;
  if (kind == kCG) {
    const float res = (float)sqrt(fmax(rr, 0.0));
    st->rr = rr;
    st->residual = res;
    if (!finite || !finite_d(rr) || !finite_f(res) || !finite_f(b_norm)) st->status = -3;
    else if (res <= tol) st->status = 0;
    else st->status = kStatusRunning;
  } else {
    const float true_rr = (float)rr;
    const float rho = (float)rz;
    const float res = __fsqrt_rn(fmaxf(true_rr, 0.0f));
    st->true_rr = true_rr;
    st->rho = rho;
    st->residual = res;
    if (!finite || !finite_f(true_rr) || !finite_f(rho)) st->status = -3;
    else if (res <= tol) st->status = 0;
    else if (rho <= 0.0f) st->status = -2;
    else st->status = kStatusRunning;
  }
  if (st->status == kStatusRunning && st->maxiter <= 0) st->status = 1;  // cg.cpp:150 / pcg.cpp:163
}

// After Ap: red = {p.Ap, p.p, Ap.Ap, nonfinite(p, Ap)}.
__device__ void decide_spmv(CgState *st, int kind) {
  const float eps = 1.1920928955078125e-07f;  // FLT_EPSILON
  const int it = st->it;
  if (kind == kCG) {
    const double denom = st->red[0];
    if (st->red[3] != 0.0 || !finite_d(denom)) {
      st->status = -3;
      st->completed = it - 1;
      return;
    }
    if (fabs(denom) <= (double)eps) {
      const double scale = sqrt(fmax(st->red[1] * st->red[2], 0.0));
      const double dtol = fmin((double)eps, (double)eps * (double)eps * fmax(1.0, scale));
      if (!finite_d(scale)) {
        st->status = -3;
        st->completed = it - 1;
        return;
      }
      if (fabs(denom) <= dtol) {
        st->status = -1;
        st->completed = it - 1;
        return;
      }
    }
    const double alpha = st->rr / denom;
    if (!finite_d(alpha)) {
      st->status = -3;
      st->completed = it - 1;
      return;
    }
    st->alpha_d = alpha;
  } else {
    const float denom = (float)st->red[0];
    const float pn = (float)st->red[1];
    const float apn = (float)st->red[2];
    const float scale = __fsqrt_rn(fmaxf(__fmul_rn(pn, apn), 0.0f));
    const float dtol = __fmul_rn(eps, fmaxf(1.0f, scale));
    if (!finite_f(denom) || !finite_f(scale) || fabsf(denom) <= dtol) {
      st->status = -1;
      st->completed = it - 1;
      return;
    }
    const float alpha = __fdiv_rn(st->rho, denom);
    if (!finite_f(alpha)) {
      st->status = -3;
      st->completed = it - 1;
      return;
    }
    st->alpha_f = alpha;
  }
}

// After the x/r update: red = {r.r, r.z, nonfinite, -}.
__device__ void decide_update(CgState *st, int kind) {
  const int it = st->it;
  st->completed = it;
  if (kind == kCG) {
    const double rr_new = st->red[0];
    const float r_norm = (float)sqrt(fmax(rr_new, 0.0));
    if (st->red[2] != 0.0 || !finite_d(rr_new) || !finite_f(r_norm)) {
      st->status = -3;
      return;
    }
    if (r_norm <= st->tol) {
      st->status = 0;
      st->rr = rr_new;
      return;
    }
    const double beta = rr_new / st->rr;
    if (!finite_d(beta)) {
      st->status = -3;
      return;
    }
    st->beta_d = beta;
    st->rr_pending = rr_new;
  } else {
    const float true_rr = (float)st->red[0];
    st->true_rr = true_rr;
    const float r_norm = __fsqrt_rn(fmaxf(true_rr, 0.0f));
    if (st->red[2] != 0.0 || !finite_f(true_rr) || !finite_f(r_norm)) {
      st->status = -3;
      return;
    }
    if (r_norm <= st->tol) {
      st->status = 0;
      return;
    }
    if (kind == kCheb) return;  // r.z needs z = p_d(M) r first (decide_rho)
    const float rho_new = (float)st->red[1];
    if (!finite_f(rho_new) || rho_new <= 0.0f) {
      st->status = -2;
      return;
    }
    const float beta = __fdiv_rn(rho_new, st->rho);
    if (!finite_f(beta)) {
      st->status = -3;
      return;
    }
    st->beta_f = beta;
    st->rho = rho_new;
    // PCG: p update cannot fail, so the iteration ends here.
    if (it >= st->maxiter) st->status = st->maxiter;
    st->it = it + 1;
  }
}

// Chebyshev PCG after z = p_d(M) r: red = {r.r, r.z, -, -}
// (chebyshev.cpp:283-297, the tail of Jacobi PCG's update).
__device__ void decide_rho(CgState *st) {
  const float rho_new = (float)st->red[1];
  if (!finite_f(rho_new) || rho_new <= 0.0f) {
    st->status = -2;
    return;
  }
  const float beta = __fdiv_rn(rho_new, st->rho);
  if (!finite_f(beta)) {
    st->status = -3;
    return;
  }
  st->beta_f = beta;
  st->rho = rho_new;
  if (st->it >= st->maxiter) st->status = st->maxiter;
  st->it = st->it + 1;
}

// Plain CG after the p update: red = {nonfinite, -, -, -}.
__device__ void decide_pupdate(CgState *st) {
  if (st->red[0] != 0.0) {
    st->status = -3;  // rr keeps its previous value (cg.cpp:238-246)
    return;
  }
  st->rr = st->rr_pending;
  if (st->it >= st->maxiter) st->status = st->maxiter;
  st->it = st->it + 1;
}

// ---- kernels ---------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads)
init_kernel(int kind, const float *__restrict__ b, const float *__restrict__ x, const float *__restrict__ ap,
            const float *__restrict__ inv_diag, float *__restrict__ r, float *__restrict__ z, float *__restrict__ p,
            int64_t n, double *partials, CgState *st, float rtol, float atol, bool decide, const P2pLink *L) {
  pdl_wait();
  pdl_trigger();
  double v[4] = {0.0, 0.0, 0.0, 0.0};
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float bi = b[i];
    const float ri = __fsub_rn(bi, ap[i]);
    v[0] += (double)bi * (double)bi;
    v[1] += (double)ri * (double)ri;
    r[i] = ri;
    if (kind == kCG) {
      p[i] = ri;
      if (!(finite_f(ri) && finite_f(ap[i]) && finite_f(bi) && finite_f(x[i]))) v[3] += 1.0;
    } else if (kind == kCheb) {
      // z = p_d(M) r and r.z follow once r is complete (chebyshev.cpp:207-222)
      if (!(finite_f(ri) && finite_f(bi) && finite_f(x[i]))) v[3] += 1.0;
    } else {
      const float inv = inv_diag[i];
      const float zi = __fmul_rn(inv, ri);
      z[i] = zi;
      p[i] = zi;
      v[2] += (double)ri * (double)zi;
      if (!(finite_f(ri) && finite_f(zi) && finite_f(inv))) v[3] += 1.0;
    }
  }
  reduce_and_decide(v, partials, st, L, decide, [&] {
    if (kind == kCheb) {
      st->bb_init = st->red[0];
      st->bad_init = st->red[3];
    } else {
      decide_init(st, kind, rtol, atol);
    }
  });
}

// Fuses p.Ap, p.p, Ap.Ap (and the non-finite count) into the SpMV row
// epilogue; the last CTA makes the step decision.
template <bool kHaloWords> struct DotsEpilogueT {
  static constexpr int kMinBlocks = 6;  // room for the fp64 accumulators
  const float *p;
  double *partials;
  CgState *st;
  int kind;
  bool decide;
  bool halo;       // peer memory: read halo columns from the halo words
  int64_t n_owned;  // halo columns start here
  const P2pLink *L;  // null: no peer exchange
  double pap, pp, apap, bad;
  static constexpr bool kHalo = kHaloWords;
  static constexpr bool kShortPipe = true;  // measured faster inside the CG iteration (256^3: 61.3 vs 64.0 ms)
  __device__ __forceinline__ bool skip() const {
    trace_start(st, 0);
    return st->status != kStatusRunning;
  }
  __device__ __forceinline__ int64_t halo_from() const { return halo ? n_owned : INT64_MAX; }
  __device__ __forceinline__ float halo_x(int64_t col) {
    return halo_read(st, L, col - n_owned, st->round_base + (unsigned)st->it);
  }
  __device__ __forceinline__ void row(int64_t r, float apv) {
    const float pv = __ldg(p + r);
    pap += (double)pv * (double)apv;
    pp += (double)pv * (double)pv;
    apap += (double)apv * (double)apv;
    if (!(finite_f(pv) && finite_f(apv))) bad += 1.0;
  }
  __device__ __forceinline__ void finish() {
    double v[4] = {pap, pp, apap, bad};
    reduce_and_decide(v, partials, st, L, decide, [&] { decide_spmv(st, kind); }, 0);
  }
};

__global__ void __launch_bounds__(kThreads)
dots_kernel(int kind, const float *__restrict__ p, const float *__restrict__ ap, int64_t n, double *partials,
            CgState *st, bool decide, const P2pLink *L) {
  pdl_wait();
  pdl_trigger();
  if (st->status != kStatusRunning) return;
  double v[4] = {0.0, 0.0, 0.0, 0.0};
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float pv = p[i], av = ap[i];
    v[0] += (double)pv * (double)av;
    v[1] += (double)pv * (double)pv;
    v[2] += (double)av * (double)av;
    if (!(finite_f(pv) && finite_f(av))) v[3] += 1.0;
  }
  reduce_and_decide(v, partials, st, L, decide, [&] { decide_spmv(st, kind); });
}

__global__ void __launch_bounds__(kThreads)
update_kernel(int kind, float *__restrict__ x, float *__restrict__ r, float *__restrict__ z,
              const float *__restrict__ p, const float *__restrict__ ap, const float *__restrict__ inv_diag,
              int64_t n, double *partials, CgState *st, bool decide, const P2pLink *L) {
  pdl_wait();
  pdl_trigger();
  trace_start(st, 1);
  if (st->status != kStatusRunning) return;
  double v[4] = {0.0, 0.0, 0.0, 0.0};
  if (kind == kCG) {
    const double alpha = st->alpha_d;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const double xc = __dadd_rn((double)x[i], __dmul_rn(alpha, (double)p[i]));
      const double rc = __dsub_rn((double)r[i], __dmul_rn(alpha, (double)ap[i]));
      const float xf = __double2float_rn(xc), rf = __double2float_rn(rc);
      if (!finite_d(xc) || !finite_d(rc) || !finite_f(xf) || !finite_f(rf)) {
        v[2] += 1.0;  // element skipped, as cg.cpp:210-214
        continue;
      }
      x[i] = xf;
      r[i] = rf;
      v[0] += (double)rf * (double)rf;
    }
  } else if (kind == kCheb) {
    const float alpha = st->alpha_f;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
      const float xo = __fadd_rn(x[i], __fmul_rn(alpha, p[i]));
      const float ro = __fsub_rn(r[i], __fmul_rn(alpha, ap[i]));
      x[i] = xo;
      r[i] = ro;
      v[0] += (double)ro * (double)ro;
      if (!(finite_f(xo) && finite_f(ro))) v[2] += 1.0;
    }
  } else {
    const float alpha = st->alpha_f;
    auto upd = [&](float xv, float pv, float rv, float av, float iv, float &xo, float &ro, float &zo) {
      xo = __fadd_rn(xv, __fmul_rn(alpha, pv));
      ro = __fsub_rn(rv, __fmul_rn(alpha, av));
      zo = __fmul_rn(iv, ro);
      v[0] += (double)ro * (double)ro;
      v[1] += (double)ro * (double)zo;
      if (!(finite_f(xo) && finite_f(ro) && finite_f(zo))) v[2] += 1.0;
    };
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t done = 0;
    if (aligned16(x) && aligned16(r) && aligned16(z) && aligned16(p) && aligned16(ap) && aligned16(inv_diag)) {
      // 16-byte vectors: 6 streams of 4 floats per thread per step
      const int64_t n4 = n / 4;
      for (int64_t i = first; i < n4; i += stride) {
        const float4 xv = reinterpret_cast<const float4 *>(x)[i], pv = __ldcs(reinterpret_cast<const float4 *>(p) + i);
        const float4 rv = reinterpret_cast<const float4 *>(r)[i], av = __ldcs(reinterpret_cast<const float4 *>(ap) + i);
        const float4 iv = __ldcs(reinterpret_cast<const float4 *>(inv_diag) + i);
        float4 xo, ro, zo;
        upd(xv.x, pv.x, rv.x, av.x, iv.x, xo.x, ro.x, zo.x);
        upd(xv.y, pv.y, rv.y, av.y, iv.y, xo.y, ro.y, zo.y);
        upd(xv.z, pv.z, rv.z, av.z, iv.z, xo.z, ro.z, zo.z);
        upd(xv.w, pv.w, rv.w, av.w, iv.w, xo.w, ro.w, zo.w);
        reinterpret_cast<float4 *>(x)[i] = xo;
        reinterpret_cast<float4 *>(r)[i] = ro;
        reinterpret_cast<float4 *>(z)[i] = zo;
      }
      done = n4 * 4;
    }
    for (int64_t i = done + first; i < n; i += stride) {
      float xo, ro, zo;
      upd(x[i], p[i], r[i], ap[i], inv_diag[i], xo, ro, zo);
      x[i] = xo;
      r[i] = ro;
      z[i] = zo;
    }
  }
  reduce_and_decide(v, partials, st, L, decide, [&] { decide_update(st, kind); }, 1);
}

// p_next = r + beta p (CG, double) or z + beta p (PCG, float), from p_cur
// (p_next == p_cur updates in place). Peer memory: the first pp->ctas CTAs
// only compute the entries the peers read (from the unchanged inputs) and
// store them straight into the peers' halo words; the remaining CTAs update
// this rank's rows, so the pushes overlap the update.
__global__ void __launch_bounds__(kThreads)
pupdate_kernel(int kind, const float *__restrict__ r, const float *__restrict__ z, const float *p_cur, float *p_next,
               int64_t n, double *partials, CgState *st, bool decide, const P2pLink *L, const PushPlan *pp) {
  pdl_wait();
  pdl_trigger();
  if (st->status != kStatusRunning) return;
  const int P = L ? push_ctas(pp) : 0;
  const bool pusher = (int)blockIdx.x < P;
  const int64_t stride = (int64_t)(gridDim.x - P) * blockDim.x;
  const int64_t first = (int64_t)(blockIdx.x - P) * blockDim.x + threadIdx.x;
  if (kind == kCG) {
    const double beta = st->beta_d;
    double v[4] = {0.0, 0.0, 0.0, 0.0};
    if (pusher) {
      // read by iteration it + 1 (decide_pupdate advances it at the end)
      halo_push(pp, st->round_base + (unsigned)st->it + 1u, [&](int i) {
        const float old = p_cur[i];
        const double pc = __dadd_rn((double)r[i], __dmul_rn(beta, (double)old));
        const float pf = __double2float_rn(pc);
        return (!finite_d(pc) || !finite_f(pf)) ? old : pf;
      });
    } else {
      for (int64_t i = first; i < n; i += stride) {
        const float old = p_cur[i];
        const double pc = __dadd_rn((double)r[i], __dmul_rn(beta, (double)old));
        const float pf = __double2float_rn(pc);
        if (!finite_d(pc) || !finite_f(pf)) {
          v[0] += 1.0;  // p keeps its value (cg.cpp:238-246)
          if (p_next != p_cur) p_next[i] = old;
          continue;
        }
        p_next[i] = pf;
      }
    }
    reduce_and_decide(v, partials, st, L, decide, [&] { decide_pupdate(st); });
    return;
  }
  const float beta = st->beta_f;
  if (pusher) {
    // decide_update already advanced it to the iteration that reads p_next
    halo_push(pp, st->round_base + (unsigned)st->it, [&](int i) { return __fadd_rn(z[i], __fmul_rn(beta, p_cur[i])); });
    return;
  }
  int64_t done = 0;
  if (aligned16(z) && aligned16(p_cur) && aligned16(p_next)) {
    const int64_t n4 = n / 4;
    for (int64_t i = first; i < n4; i += stride) {
      const float4 zv = __ldcs(reinterpret_cast<const float4 *>(z) + i);
      float4 pv = reinterpret_cast<const float4 *>(p_cur)[i];
      pv.x = __fadd_rn(zv.x, __fmul_rn(beta, pv.x));
      pv.y = __fadd_rn(zv.y, __fmul_rn(beta, pv.y));
      pv.z = __fadd_rn(zv.z, __fmul_rn(beta, pv.z));
      pv.w = __fadd_rn(zv.w, __fmul_rn(beta, pv.w));
      reinterpret_cast<float4 *>(p_next)[i] = pv;
    }
    done = n4 * 4;
  }
  for (int64_t i = done + first; i < n; i += stride) p_next[i] = __fadd_rn(z[i], __fmul_rn(beta, p_cur[i]));
}

// r.r and r.z after the Chebyshev apply; at the start (`first`) also p = z
// and the initial decision, in the solve loop the rho / beta decision.
__global__ void __launch_bounds__(kThreads)
cheb_dots_kernel(const float *__restrict__ r, const float *__restrict__ z, float *__restrict__ p, int64_t n,
                 double *partials, CgState *st, bool first, float rtol, float atol) {
  if (st->status != kStatusRunning) return;
  double v[4] = {0.0, 0.0, 0.0, 0.0};
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float rv = r[i], zv = z[i];
    v[0] += (double)rv * (double)rv;
    v[1] += (double)rv * (double)zv;
    if (first) p[i] = zv;
  }
  reduce_and_decide(v, partials, st, nullptr, true, [&] {
    if (first) {
      const double rr = st->red[0], rz = st->red[1];
      st->red[0] = st->bb_init;
      st->red[1] = rr;
      st->red[2] = rz;
      st->red[3] = st->bad_init;
      decide_init(st, kPCG, rtol, atol);
    } else {
      decide_rho(st);
    }
  });
}

// Chebyshev semi-iteration (chebyshev.cpp:84-122): out = scale * rhs, then
// per step next = (1 - w) prev + w out + w scale (rhs - M out). The kernels
// return at once when a solve has stopped (st may be null: standalone).
__global__ void cheb_first_kernel(const CgState *st, const float *__restrict__ rhs, float *__restrict__ out,
                                  float *__restrict__ prev, int64_t n, float scale) {
  if (st && st->status != kStatusRunning) return;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    out[i] = __fmul_rn(scale, rhs[i]);
    if (prev) prev[i] = 0.0f;
  }
}

__global__ void cheb_step_kernel(const CgState *st, const float *__restrict__ rhs, const float *__restrict__ ax,
                                 const float *__restrict__ prev, const float *__restrict__ out,
                                 float *__restrict__ next, int64_t n, float one_minus_omega, float omega,
                                 float omega_scale) {
  if (st && st->status != kStatusRunning) return;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float rv = __fsub_rn(rhs[i], ax[i]);
    next[i] = __fadd_rn(__fadd_rn(__fmul_rn(one_minus_omega, prev[i]), __fmul_rn(omega, out[i])),
                        __fmul_rn(omega_scale, rv));
  }
}

// SpMV epilogue that only stores y and skips the launch once the solve stopped.
struct StatusSkipEpilogue : NoEpilogue {
  const CgState *st;
  __device__ __forceinline__ bool skip() const { return st && st->status != kStatusRunning; }
};

// Multi-GPU: the reductions leave local sums in st->red; after the NCCL
// all-reduce one thread makes the decision every rank makes identically.
__global__ void decide_kernel(CgState *st, int which, int kind, float rtol, float atol) {
  if (which != 0 && st->status != kStatusRunning) return;
  switch (which) {
  case 0: decide_init(st, kind, rtol, atol); break;
  case 1: decide_spmv(st, kind); break;
  case 2: decide_update(st, kind); break;
  default: decide_pupdate(st); break;
  }
}

__global__ void halo_pack_kernel(const float *__restrict__ v, const int *__restrict__ idx, float *__restrict__ out,
                                 int64_t n) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) out[i] = v[idx[i]];
}

// Standalone halo push of v's send entries as round `round` (x0 and the first
// direction; the iterations push from the direction update).
__global__ void p2p_halo_push_kernel(CgState *st, const float *__restrict__ v, const PushPlan *pp, int round) {
  if (st->status != kStatusRunning) return;
  halo_push(pp, st->round_base + (unsigned)round, [&](int i) { return v[i]; });
}

// Copies the halo words of a round (round < 0: the current iteration's) into
// the halo part of a vector, for SpMV kernels that do not read the words
// themselves.
__global__ void p2p_halo_unpack_kernel(CgState *st, const P2pLink *L, float *__restrict__ v_halo, int64_t n_halo,
                                       int round) {
  if (st->status != kStatusRunning) return;
  const unsigned r = st->round_base + (unsigned)(round >= 0 ? round : st->it);
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < n_halo; j += (int64_t)gridDim.x * blockDim.x)
    v_halo[j] = halo_read(st, L, j, r);
}

int elementwise_grid(int64_t n) {
  static thread_local int dev_cached = -1, sms = 0;
  int dev = 0;
  MSX_CUDA(cudaGetDevice(&dev));
  if (dev != dev_cached) {
    sms = num_sms();
    dev_cached = dev;
  }
  const int64_t want = ceil_div(n, kThreads);
  const int64_t cap = (int64_t)sms * 8;
  return (int)std::max<int64_t>(1, std::min(want, cap));
}

}  // namespace

struct CgEngine {
  CgEngineConfig cfg{};
  int kind = kCG;
  int64_t n = 0, n_cols = 0;
  int device = 0;
  BinnedPlan plan;
  bool fused = true;
  int red_grid = 1;
  void *plan_mem = nullptr;
  void *mem = nullptr;       // state, partials, vectors (one allocation)
  float *pbuf = nullptr;     // direction buffer(s)
  float *p[2] = {};          // P2P: two buffers, alternating by iteration parity; else p[0] == p[1]
  unsigned long long *halo_words = nullptr;  // P2P: own allocation, IPC-exported
  unsigned round_base = 1;   // P2P: halo round 0 of the next solve (identical on every rank)
  int64_t p_stride = 0;      // elements between p[0] and p[1]
  Mailbox *mbox = nullptr;   // own allocation (IPC-exported in P2P mode)
  CgState *st = nullptr;
  CommState *cs = nullptr;
  double *partials = nullptr;
  float *carry = nullptr, *r = nullptr, *z = nullptr, *ap = nullptr, *x = nullptr, *b = nullptr, *inv = nullptr;
  float *sendbuf = nullptr;
  int64_t n_send = 0;
  // P2P
  P2pLink link{};            // host copy
  PushPlan push{};           // host copy
  P2pLink *link_dev = nullptr;   // device copies (P2P only)
  PushPlan *push_dev = nullptr;
  int push_grid = 1;
  void *opened[2 * kMaxRanks] = {};
  bool connected = false;
  cudaStream_t s = nullptr;
  cudaEvent_t ev = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int batch = 4;
  bool pdl = false;          // programmatic dependent launch inside the iteration graph (MSX_CG_PDL=1)
  int *status_host = nullptr;  // two slots (batches in flight)
  cudaEvent_t batch_done[2] = {};
  // Chebyshev preconditioner: plan of M, its chunk carry, the three
  // semi-iteration buffers and the host-computed step coefficients
  BinnedPlan plan_m;
  void *plan_m_mem = nullptr;
  float *carry_m = nullptr;
  float *cheb[3] = {};
  float cheb_scale = 0.f;
  std::vector<float> cheb_coef;  // per step: 1 - omega, omega, omega * scale
};

namespace {

bool p2p(const CgEngine *e) { return e->cfg.comm == kCommP2p; }
const P2pLink *link_of(const CgEngine *e) { return p2p(e) ? e->link_dev : nullptr; }
const PushPlan *push_of(const CgEngine *e) { return p2p(e) ? e->push_dev : nullptr; }

// NCCL halo exchange of v (owned part -> peers' halo part).
void engine_exchange_nccl(CgEngine *e, float *v, cudaStream_t q) {
  const CgEngineConfig &c = e->cfg;
#if defined(MSX_HAVE_NCCL)
  if (c.comm != kCommNccl) return;
  if (e->n_send > 0) {
    halo_pack_kernel<<<(unsigned)ceil_div(e->n_send, 256), 256, 0, q>>>(v, c.send_idx, e->sendbuf, e->n_send);
    MSX_CHECK_LAUNCH();
  }
  ncclComm_t comm = static_cast<ncclComm_t>(c.nccl_comm);
  auto nccl = [](ncclResult_t r) {
    if (r != ncclSuccess) fail(MSX_ERR_RUNTIME, std::string("NCCL: ") + ncclGetErrorString(r));
  };
  nccl(ncclGroupStart());
  int64_t so = 0, ro = 0;
  for (int k = 0; k < c.n_peers; ++k) {
    if (c.send_counts[k] > 0)
      nccl(ncclSend(e->sendbuf + so, (size_t)c.send_counts[k], ncclFloat, c.peers[k], comm, q));
    if (c.recv_counts[k] > 0)
      nccl(ncclRecv(v + e->n + ro, (size_t)c.recv_counts[k], ncclFloat, c.peers[k], comm, q));
    so += c.send_counts[k];
    ro += c.recv_counts[k];
  }
  nccl(ncclGroupEnd());
#else
  (void)v;
  (void)q;
  if (c.comm == kCommNccl) fail(MSX_ERR_RUNTIME, "this build has no NCCL.");
#endif
}

// Peer memory: push v's send entries into the peers' halo words as `round`.
void engine_push(CgEngine *e, const float *v, int round, cudaStream_t q) {
  p2p_halo_push_kernel<<<e->push_grid, kThreads, 0, q>>>(e->st, v, push_of(e), round);
  MSX_CHECK_LAUNCH();
}

// Peer memory: copy the halo words of `round` (< 0: the current iteration's)
// into v's halo part.
void engine_unpack(CgEngine *e, float *v, int round, cudaStream_t q) {
  const int64_t nh = e->cfg.n_halo;
  if (nh == 0) return;
  p2p_halo_unpack_kernel<<<(unsigned)std::min<int64_t>(ceil_div(nh, kThreads), 1024), kThreads, 0, q>>>(
      e->st, link_of(e), v + e->n, nh, round);
  MSX_CHECK_LAUNCH();
}

// NCCL: after a reduction kernel left local sums in st->red, all-reduce them
// and decide. Peer memory and single GPU: the kernel's last CTA already did.
void engine_reduce_decide_nccl(CgEngine *e, int which, float rtol, float atol, cudaStream_t q) {
#if defined(MSX_HAVE_NCCL)
  const CgEngineConfig &c = e->cfg;
  if (c.comm != kCommNccl) return;
  ncclResult_t r = ncclAllReduce(e->st->red, e->st->red, 4, ncclDouble, ncclSum, static_cast<ncclComm_t>(c.nccl_comm), q);
  if (r != ncclSuccess) fail(MSX_ERR_RUNTIME, std::string("NCCL: ") + ncclGetErrorString(r));
  decide_kernel<<<1, 1, 0, q>>>(e->st, which, e->kind, rtol, atol);
  MSX_CHECK_LAUNCH();
#else
  (void)e;
  (void)which;
  (void)rtol;
  (void)atol;
  (void)q;
#endif
}

// z = p_d(M) r into e->z (chebyshev.cpp:84-122). The buffer that ends up
// holding the result depends only on the degree, so e->z is fixed at setup.
void engine_cheb_apply(CgEngine *e, cudaStream_t q) {
  const CgEngineConfig &c = e->cfg;
  const int g = elementwise_grid(e->n);
  float *out = e->cheb[0], *prev = e->cheb[1], *next = e->cheb[2];
  cheb_first_kernel<<<g, kThreads, 0, q>>>(e->st, e->r, out, c.degree > 1 ? prev : nullptr, e->n, e->cheb_scale);
  MSX_CHECK_LAUNCH();
  for (int it = 1; it < c.degree; ++it) {
    dispatch_index(c.index_dtype, [&](auto ityp) {
      using I = decltype(ityp);
      StatusSkipEpilogue epi{};
      epi.st = e->st;
      launch_spmv_binned<float, I, StatusSkipEpilogue>(e->plan_m, c.m_data, static_cast<const I *>(c.m_indices),
                                                       static_cast<const I *>(c.m_indptr), out, e->ap, e->carry_m,
                                                       epi, q);
    });
    launch_spmv_long_fixup<float>(e->plan_m, e->carry_m, e->ap, q);
    const float *k = &e->cheb_coef[3 * (it - 1)];
    cheb_step_kernel<<<g, kThreads, 0, q>>>(e->st, e->r, e->ap, prev, out, next, e->n, k[0], k[1], k[2]);
    MSX_CHECK_LAUNCH();
    float *t = prev;
    prev = out;
    out = next;
    next = t;
  }
}

// One iteration reading direction buffer `par` and writing `par ^ 1` (the
// same buffer unless P2P). Single GPU and P2P: three kernels, the scalar
// all-reduce and the halo exchange fused into them.
void engine_iteration(CgEngine *e, int par, cudaStream_t q) {
  const CgEngineConfig &c = e->cfg;
  const bool decide = c.comm == kCommNone;
  const int kind = e->kind;
  // kernels follow kernels directly (no NCCL call in between): overlap launches
  const bool pdl = c.comm != kCommNccl && e->pdl;
  float *pc = e->p[par], *pn = e->p[par ^ 1];
  engine_exchange_nccl(e, pc, q);
  // the short-row SpMV reads the halo words itself; other kernels get them unpacked
  // The halo words are unpacked into p's halo slots by a small kernel before
  // the SpMV (default): reading them inside the SpMV (MSX_CG_HALO_IN_SPMV=1)
  // slowed its gathers (2 GPUs, 8.4 M rows each: 149 us against 131 us plus
  // a 2.4 us unpack).
  static const int halo_in_spmv = [] {
    const char *v = std::getenv("MSX_CG_HALO_IN_SPMV");
    return v && *v ? std::atoi(v) : 0;
  }();
  const bool words_in_spmv = p2p(e) && e->fused && short_rows_plan(e->plan) && halo_in_spmv != 0;
  if (p2p(e) && !words_in_spmv) engine_unpack(e, pc, -1, q);
  if (e->fused) {
    dispatch_index(c.index_dtype, [&](auto ityp) {
      using I = decltype(ityp);
      auto run = [&](auto epi) {
        launch_spmv_binned<float, I, decltype(epi)>(e->plan, c.data, static_cast<const I *>(c.indices),
                                                    static_cast<const I *>(c.indptr), pc, e->ap, e->carry, epi, q, pdl);
      };
      if (words_in_spmv)
        run(DotsEpilogueT<true>{pc, e->partials, e->st, kind, decide, true, e->n, link_of(e), 0.0, 0.0, 0.0, 0.0});
      else
        run(DotsEpilogueT<false>{pc, e->partials, e->st, kind, decide, false, e->n, link_of(e), 0.0, 0.0, 0.0, 0.0});
    });
  } else {
    spmv_binned_run(MSX_F32, c.index_dtype, e->plan, c.data, c.indices, c.indptr, pc, e->ap, e->carry, q);
    dots_kernel<<<e->red_grid, kThreads, 0, q>>>(kind, pc, e->ap, e->n, e->partials, e->st, decide, link_of(e));
    MSX_CHECK_LAUNCH();
  }
  engine_reduce_decide_nccl(e, 1, 0.f, 0.f, q);
  launch(update_kernel, dim3(e->red_grid), dim3(kThreads), 0, q, pdl, kind, e->x, e->r, e->z, pc, e->ap, e->inv, e->n,
         e->partials, e->st, decide, link_of(e));
  engine_reduce_decide_nccl(e, 2, 0.f, 0.f, q);
  if (kind == kCheb) {
    engine_cheb_apply(e, q);
    cheb_dots_kernel<<<e->red_grid, kThreads, 0, q>>>(e->r, e->z, nullptr, e->n, e->partials, e->st, false, 0.f, 0.f);
    MSX_CHECK_LAUNCH();
  }
  launch(pupdate_kernel, dim3(e->red_grid + (p2p(e) ? e->push_grid : 0)), dim3(kThreads), 0, q, pdl, kind, e->r, e->z,
         pc, pn, e->n, e->partials, e->st, decide, link_of(e), push_of(e));
  if (kind == kCG) engine_reduce_decide_nccl(e, 3, 0.f, 0.f, q);
}

template <typename T> T *bump(char *&cur, size_t count) {
  T *p = reinterpret_cast<T *>(cur);
  cur += (sizeof(T) * count + 255) & ~size_t(255);
  return p;
}

// Layout of one rank's peer-memory descriptor.
struct IpcBlob {
  cudaIpcMemHandle_t halo;
  cudaIpcMemHandle_t mbox;
  int64_t n_owned;
};
static_assert(sizeof(IpcBlob) <= kCgIpcBytes, "descriptor too large");

}  // namespace

CgEngine *cg_engine_create(const CgEngineConfig &cfg, cudaStream_t user_stream) {
  if (cfg.world > kMaxRanks) fail(MSX_ERR_INVALID, "CG: at most 8 ranks (one node).");
#if !defined(MSX_HAVE_NCCL)
  if (cfg.comm == kCommNccl) fail(MSX_ERR_RUNTIME, "this build has no NCCL: multi-GPU CG over NCCL is unavailable.");
#endif
  // destroyed (buffers freed) if anything below throws
  std::unique_ptr<CgEngine, void (*)(CgEngine *)> e(new CgEngine(), cg_engine_destroy);
  CgEngine *E = e.get();
  E->cfg = cfg;
  E->kind = cfg.m_data ? kCheb : (cfg.preconditioned ? kPCG : kCG);
  if (E->kind == kCheb && cfg.comm != kCommNone)
    fail(MSX_ERR_INVALID, "Chebyshev-preconditioned CG runs on one GPU.");
  E->n = cfg.n;
  E->n_cols = cfg.n + cfg.n_halo;
  MSX_CUDA(cudaGetDevice(&E->device));
  MSX_CUDA(cudaStreamCreateWithFlags(&E->s, cudaStreamNonBlocking));
  MSX_CUDA(cudaEventCreateWithFlags(&E->ev, cudaEventDisableTiming));
  MSX_CUDA(cudaEventRecord(E->ev, user_stream));
  MSX_CUDA(cudaStreamWaitEvent(E->s, E->ev, 0));
  cudaStream_t s = E->s;
  build_binned_plan(cfg.index_dtype, cfg.indptr, E->n, cfg.nnz, s,
                    [&](size_t bytes) -> void * {
                      MSX_CUDA(cudaMalloc(&E->plan_mem, bytes));
                      return E->plan_mem;
                    },
                    E->plan);
  E->fused = E->plan.n_long == 0;
  if (E->kind == kCheb) {
    build_binned_plan(cfg.index_dtype, cfg.m_indptr, E->n, cfg.m_nnz, s,
                      [&](size_t bytes) -> void * {
                        MSX_CUDA(cudaMalloc(&E->plan_m_mem, bytes));
                        return E->plan_m_mem;
                      },
                      E->plan_m);
    // step coefficients in the reference's float arithmetic (chebyshev.cpp:89-114)
    const float lmin = cfg.lambda_min, lmax = cfg.lambda_max;
    const float scale = 2.0f / (lmax + lmin);
    const float alpha = 1.0f - scale * lmin;
    const float mu = 1.0f / alpha;
    const float omega_prod = 2.0f / alpha;
    float c_prev = 1.0f, c_cur = mu;
    E->cheb_scale = scale;
    for (int it = 1; it < cfg.degree; ++it) {
      const float c_next = 2.0f * mu * c_cur - c_prev;
      const float omega = omega_prod * c_cur / c_next;
      E->cheb_coef.push_back(1.0f - omega);
      E->cheb_coef.push_back(omega);
      E->cheb_coef.push_back(omega * scale);
      c_prev = c_cur;
      c_cur = c_next;
    }
  }
  E->red_grid = elementwise_grid(E->n);
  int64_t spmv_grid_n = 0;
  dispatch_index(cfg.index_dtype, [&](auto ityp) {
    using I = decltype(ityp);
    spmv_grid_n = std::max({binned_grid<float, I, DotsEpilogueT<true>>(E->plan),
                            binned_grid<float, I, DotsEpilogueT<false>>(E->plan),
                            binned_grid<float, I, NoEpilogue>(E->plan)});
  });
  for (int k = 0; k < cfg.n_peers; ++k) E->n_send += cfg.send_counts[k];
  // pushing CTAs: about 512 entries each (MSX_P2P_PUSH_PER_CTA overrides)
  int64_t per_cta = 2 * kThreads;
  if (const char *v = std::getenv("MSX_P2P_PUSH_PER_CTA")) per_cta = std::max<int64_t>(kThreads, std::atoll(v));
  E->push_grid = (int)std::min<int64_t>(std::max<int64_t>(ceil_div(E->n_send, per_cta), 1), E->red_grid);
  const int64_t max_grid = std::max<int64_t>(E->red_grid + E->push_grid, spmv_grid_n);
  const size_t vec = (size_t)std::max<int64_t>(E->n, 1);
  size_t bytes = 0;
  auto sz = [](size_t b) { return (b + 255) & ~size_t(255); };
  bytes += sz(sizeof(CgState)) + sz(sizeof(CommState)) + sz(sizeof(double) * 4 * max_grid) +
           sz(sizeof(float) * std::max<int64_t>(E->plan.n_chunks, 1)) +
           sz(sizeof(float) * std::max<int64_t>(E->plan_m.n_chunks, 1)) + 9 * sz(sizeof(float) * vec) +
           sz(sizeof(float) * std::max<int64_t>(E->n_send, 1)) + sz(sizeof(P2pLink)) + sz(sizeof(PushPlan));
  MSX_CUDA(cudaMalloc(&E->mem, bytes));
  MSX_CUDA(cudaMemsetAsync(E->mem, 0, bytes, s));
  char *cur = static_cast<char *>(E->mem);
  E->st = bump<CgState>(cur, 1);
  E->cs = bump<CommState>(cur, 1);
  E->partials = bump<double>(cur, 4 * max_grid);
  E->carry = bump<float>(cur, std::max<int64_t>(E->plan.n_chunks, 1));
  E->carry_m = bump<float>(cur, std::max<int64_t>(E->plan_m.n_chunks, 1));
  for (float *&c : E->cheb) c = bump<float>(cur, vec);
  E->r = bump<float>(cur, vec);
  E->z = bump<float>(cur, vec);
  E->ap = bump<float>(cur, vec);
  E->x = bump<float>(cur, vec);
  E->b = bump<float>(cur, vec);
  E->inv = bump<float>(cur, vec);
  E->sendbuf = bump<float>(cur, std::max<int64_t>(E->n_send, 1));
  E->link_dev = bump<P2pLink>(cur, 1);
  E->push_dev = bump<PushPlan>(cur, 1);
  // direction buffers: two (16-byte aligned apart) in P2P mode
  const int64_t cols = std::max<int64_t>(E->n_cols, 1);
  const bool dbl = cfg.comm == kCommP2p;
  E->p_stride = dbl ? (cols + 63) / 64 * 64 : 0;
  const int64_t p_elems = dbl ? 2 * E->p_stride : cols;
  MSX_CUDA(cudaMalloc(&E->pbuf, sizeof(float) * (size_t)p_elems));
  MSX_CUDA(cudaMemsetAsync(E->pbuf, 0, sizeof(float) * (size_t)p_elems, s));
  E->p[0] = E->pbuf;
  E->p[1] = E->pbuf + E->p_stride;
  MSX_CUDA(cudaMalloc(&E->mbox, sizeof(Mailbox)));
  MSX_CUDA(cudaMemsetAsync(E->mbox, 0, sizeof(Mailbox), s));
  if (cfg.comm == kCommP2p) {
    const size_t hb = sizeof(unsigned long long) * (size_t)std::max<int64_t>(cfg.n_halo, 1);
    MSX_CUDA(cudaMalloc(&E->halo_words, hb));
    MSX_CUDA(cudaMemsetAsync(E->halo_words, 0, hb, s));  // flag 0: no round (rounds start at 1)
  }
  if (E->kind == kCheb) {
    // the semi-iteration rotates (out, prev, next) once per step
    const int d = std::max(cfg.degree, 1);
    const int final_slot[3] = {0, 2, 1};  // out after (d - 1) rotations
    E->z = E->cheb[final_slot[(d - 1) % 3]];
    E->inv = nullptr;
  } else if (!cfg.preconditioned) {
    E->z = nullptr, E->inv = nullptr;
  }
  MSX_CUDA(cudaMallocHost(&E->status_host, 2 * sizeof(int)));
  for (auto &ev : E->batch_done) MSX_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  E->link.world = 1;
  E->link.rank = 0;
  E->link.cs = E->cs;
  E->link.mine = E->mbox;
  if (cfg.comm == kCommP2p) {
    E->link.world = cfg.world;
    E->link.rank = cfg.rank;
    E->link.halo = E->halo_words;
    E->link.n_owned = E->n;
  }
  // Iterations per graph launch: about a millisecond of work per batch, even
  // (P2P alternates the direction buffers).
  const double bytes_per_iter = 8.0 * cfg.nnz + 56.0 * E->n;
  int batch = (int)std::max(1.0, std::min(64.0, 5.0e9 * 1e-3 / std::max(bytes_per_iter, 1.0)));
  E->batch = std::max(4, (batch + 1) & ~1);
  if (const char *v = std::getenv("MSX_CG_PDL")) E->pdl = std::atoi(v) != 0;
  MSX_CUDA(cudaStreamSynchronize(s));
  return e.release();
}

void cg_engine_destroy(CgEngine *e) {
  if (!e) return;
  int cur = 0;
  cudaGetDevice(&cur);
  if (cur != e->device) cudaSetDevice(e->device);
  if (e->s) cudaStreamSynchronize(e->s);
  if (e->exec) cudaGraphExecDestroy(e->exec);
  if (e->graph) cudaGraphDestroy(e->graph);
  for (void *p : e->opened)
    if (p) cudaIpcCloseMemHandle(p);
  if (e->status_host) cudaFreeHost(e->status_host);
  for (auto ev : e->batch_done)
    if (ev) cudaEventDestroy(ev);
  if (e->pbuf) cudaFree(e->pbuf);
  if (e->halo_words) cudaFree(e->halo_words);
  if (e->mbox) cudaFree(e->mbox);
  if (e->mem) cudaFree(e->mem);
  if (e->plan_mem) cudaFree(e->plan_mem);
  if (e->plan_m_mem) cudaFree(e->plan_m_mem);
  if (e->ev) cudaEventDestroy(e->ev);
  if (e->s) cudaStreamDestroy(e->s);
  if (cur != e->device) cudaSetDevice(cur);
  delete e;
}

void cg_engine_ipc_handles(CgEngine *e, void *out) {
  if (!p2p(e)) fail(MSX_ERR_INVALID, "CG context: IPC handles are for the peer-memory mode.");
  IpcBlob blob{};
  MSX_CUDA(cudaIpcGetMemHandle(&blob.halo, e->halo_words));
  MSX_CUDA(cudaIpcGetMemHandle(&blob.mbox, e->mbox));
  blob.n_owned = e->n;
  std::memset(out, 0, kCgIpcBytes);
  std::memcpy(out, &blob, sizeof(blob));
}

void cg_engine_connect(CgEngine *e, const void *all_handles) {
  const CgEngineConfig &c = e->cfg;
  if (c.comm != kCommP2p) fail(MSX_ERR_INVALID, "CG context: connect is for the peer-memory mode.");
  if (e->connected) fail(MSX_ERR_INVALID, "CG context: already connected.");
  const char *raw = static_cast<const char *>(all_handles);
  unsigned long long *hw[kMaxRanks] = {};
  int64_t owned[kMaxRanks] = {};
  for (int q = 0; q < c.world; ++q) {
    IpcBlob blob;
    std::memcpy(&blob, raw + (size_t)q * kCgIpcBytes, sizeof(blob));
    owned[q] = blob.n_owned;
    if (q == c.rank) {
      e->link.peer[q] = e->mbox;
      hw[q] = e->halo_words;
      continue;
    }
    void *hp = nullptr, *mb = nullptr;
    MSX_CUDA(cudaIpcOpenMemHandle(&hp, blob.halo, cudaIpcMemLazyEnablePeerAccess));
    e->opened[2 * q] = hp;
    MSX_CUDA(cudaIpcOpenMemHandle(&mb, blob.mbox, cudaIpcMemLazyEnablePeerAccess));
    e->opened[2 * q + 1] = mb;
    e->link.peer[q] = static_cast<Mailbox *>(mb);
    hw[q] = static_cast<unsigned long long *>(hp);
  }
  PushPlan pp{};
  long long off = 0;
  int np = 0;
  for (int k = 0; k < c.n_peers; ++k) {
    if (c.send_counts[k] == 0) continue;
    const int q = c.peers[k];
    const int64_t h0 = c.peer_dst_offset[k] - owned[q];  // first halo slot of this rank's block at q
    if (h0 < 0) fail(MSX_ERR_INVALID, "CG context: a landing offset lies inside the peer's owned rows.");
    pp.dst[np] = hw[q] + h0;
    pp.off[np] = off;
    off += c.send_counts[k];
    ++np;
  }
  pp.off[np] = off;
  pp.n_peers = np;
  pp.ctas = e->push_grid;
  pp.idx = c.send_idx;
  e->push = pp;
  MSX_CUDA(cudaMemcpyAsync(e->link_dev, &e->link, sizeof(P2pLink), cudaMemcpyHostToDevice, e->s));
  MSX_CUDA(cudaMemcpyAsync(e->push_dev, &e->push, sizeof(PushPlan), cudaMemcpyHostToDevice, e->s));
  MSX_CUDA(cudaStreamSynchronize(e->s));
  e->connected = true;
}

CgResult cg_engine_solve(CgEngine *e, const float *b_in, const float *x0_in, const float *inv_in, float *x_out,
                         float rtol, float atol, int maxiter, cudaStream_t user_stream) {
  const CgEngineConfig &c = e->cfg;
  if (p2p(e) && !e->connected) fail(MSX_ERR_RUNTIME, "CG context: peers are not connected.");
  cudaStream_t s = e->s;
  const int64_t n = e->n;
  const bool decide = c.comm == kCommNone;
  MSX_CUDA(cudaEventRecord(e->ev, user_stream));
  MSX_CUDA(cudaStreamWaitEvent(s, e->ev, 0));
  MSX_CUDA(cudaMemcpyAsync(e->b, b_in, sizeof(float) * n, cudaMemcpyDeviceToDevice, s));
  MSX_CUDA(cudaMemcpyAsync(e->x, x0_in, sizeof(float) * n, cudaMemcpyDeviceToDevice, s));
  MSX_CUDA(cudaMemcpyAsync(e->p[0], x0_in, sizeof(float) * n, cudaMemcpyDeviceToDevice, s));
  if (e->kind == kPCG) MSX_CUDA(cudaMemcpyAsync(e->inv, inv_in, sizeof(float) * n, cudaMemcpyDeviceToDevice, s));
  CgState init{};
  init.status = kStatusRunning;
  init.it = 1;
  init.maxiter = maxiter;
  init.round_base = e->round_base;
  static const bool tracing = [] {
    const char *v = std::getenv("MSX_CG_TRACE");
    return v && *v == '1';
  }();
  init.tracing = tracing ? 1 : 0;
  init.k_start[0] = init.k_start[1] = ~0ull;
  MSX_CUDA(cudaMemcpyAsync(e->st, &init, sizeof(CgState), cudaMemcpyHostToDevice, s));

  // r0 = b - A x0 (x0 staged in p[0], whose halo the exchange fills); p[0]
  // then holds the first direction, whose halo is pushed before iteration 1.
  if (p2p(e)) {
    engine_push(e, e->p[0], 0, s);
    engine_unpack(e, e->p[0], 0, s);
  }
  engine_exchange_nccl(e, e->p[0], s);
  spmv_binned_run(MSX_F32, c.index_dtype, e->plan, c.data, c.indices, c.indptr, e->p[0], e->ap, e->carry, s);
  init_kernel<<<e->red_grid, kThreads, 0, s>>>(e->kind, e->b, e->x, e->ap, e->inv, e->r, e->z, e->p[0], n,
                                               e->partials, e->st, rtol, atol, decide, link_of(e));
  MSX_CHECK_LAUNCH();
  engine_reduce_decide_nccl(e, 0, rtol, atol, s);
  if (e->kind == kCheb) {  // z0 = p_d(M) r0, p0 = z0, then the initial decision
    engine_cheb_apply(e, s);
    cheb_dots_kernel<<<e->red_grid, kThreads, 0, s>>>(e->r, e->z, e->p[0], n, e->partials, e->st, true, rtol, atol);
    MSX_CHECK_LAUNCH();
  }
  if (p2p(e)) engine_push(e, e->p[0], 1, s);  // read by iteration 1
  CgState host{};
  MSX_CUDA(cudaMemcpyAsync(&host, e->st, sizeof(CgState), cudaMemcpyDeviceToHost, s));
  MSX_CUDA(cudaStreamSynchronize(s));

  if (host.status == kStatusRunning) {
    if (!e->exec) {
      MSX_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      try {
        for (int k = 0; k < e->batch; ++k) engine_iteration(e, k & 1, s);
      } catch (...) {
        cudaGraph_t g = nullptr;
        cudaStreamEndCapture(s, &g);
        if (g) cudaGraphDestroy(g);
        throw;
      }
      MSX_CUDA(cudaStreamEndCapture(s, &e->graph));
      MSX_CUDA(cudaGraphInstantiate(&e->exec, e->graph, 0));
    }
    // Two batches in flight: while the host reads the status after batch k,
    // batch k + 1 already runs, so the GPU never waits for the host. A batch
    // launched after the solve stopped costs only its kernels' early exits
    // (identically on every rank, whose statuses agree).
    int64_t launched = 0;
    int slot = 0;
    auto launch_batch = [&](int sl) {
      MSX_CUDA(cudaGraphLaunch(e->exec, s));
      launched += e->batch;
      MSX_CUDA(cudaMemcpyAsync(e->status_host + sl, &e->st->status, sizeof(int), cudaMemcpyDeviceToHost, s));
      MSX_CUDA(cudaEventRecord(e->batch_done[sl], s));
    };
    launch_batch(0);
    while (true) {
      const bool more = launched < maxiter;
      if (more) launch_batch(slot ^ 1);
      MSX_CUDA(cudaEventSynchronize(e->batch_done[slot]));
      if (e->status_host[slot] != kStatusRunning || !more) break;
      slot ^= 1;
    }
    MSX_CUDA(cudaMemcpyAsync(&host, e->st, sizeof(CgState), cudaMemcpyDeviceToHost, s));
    MSX_CUDA(cudaStreamSynchronize(s));
  }
  if (host.tracing) {
    auto avg = [&](int k) { return host.trace[k] / 1000.0 / std::max<unsigned long long>(host.trace[k % 3 == 2 ? k : k + (2 - k % 3)], 1); };
    std::fprintf(stderr,
                 "[msx cg trace] rank %d: spmv+dots start->last CTA %.1f us, all-reduce %.1f us; update start->last "
                 "CTA %.1f us, all-reduce %.1f us (%llu iterations)\n",
                 c.rank, avg(0), avg(1), avg(3), avg(4), host.trace[2]);
  }
  // rounds 0 .. completed + 1 were used; the next solve starts past them
  e->round_base += (unsigned)host.completed + 3u;
  MSX_CUDA(cudaMemcpyAsync(x_out, e->x, sizeof(float) * n, cudaMemcpyDeviceToDevice, s));
  MSX_CUDA(cudaEventRecord(e->ev, s));
  MSX_CUDA(cudaStreamWaitEvent(user_stream, e->ev, 0));
  if (host.status == -4) fail(MSX_ERR_RUNTIME, "CG: a peer did not answer (communication timeout).");
  if (host.status == kStatusRunning) fail(MSX_ERR_RUNTIME, "CG solve ended without a status (internal error).");
  CgResult res{};
  res.info = host.status;
  res.iterations = host.completed;
  res.residual = e->kind == kCG ? (float)std::sqrt(std::max(host.rr, 0.0)) : std::sqrt(std::max(host.true_rr, 0.0f));
  return res;
}

CgResult cg_solve(const CgProblem &prob, cudaStream_t user_stream) {
  CgEngineConfig cfg{};
  cfg.index_dtype = prob.index_dtype;
  cfg.data = prob.data;
  cfg.indices = prob.indices;
  cfg.indptr = prob.indptr;
  cfg.nnz = prob.nnz;
  cfg.n = prob.n;
  cfg.n_halo = prob.n_cols - prob.n;
  cfg.preconditioned = prob.inv_diag != nullptr;
  cfg.m_data = prob.m_data;
  cfg.m_indices = prob.m_indices;
  cfg.m_indptr = prob.m_indptr;
  cfg.m_nnz = prob.m_nnz;
  cfg.degree = prob.degree;
  cfg.lambda_min = prob.lambda_min;
  cfg.lambda_max = prob.lambda_max;
  cfg.comm = kCommNone;
  cfg.rank = 0;
  cfg.world = 1;
  if (prob.dist) {
    cfg.comm = kCommNccl;
    cfg.nccl_comm = prob.dist->comm;
    cfg.n_peers = prob.dist->n_peers;
    cfg.peers = prob.dist->peers;
    cfg.send_counts = prob.dist->send_counts;
    cfg.recv_counts = prob.dist->recv_counts;
    cfg.send_idx = prob.dist->send_idx;
  }
  CgEngine *e = cg_engine_create(cfg, user_stream);
  struct Guard {
    CgEngine *e;
    ~Guard() { cg_engine_destroy(e); }
  } guard{e};
  return cg_engine_solve(e, prob.b, prob.x0, prob.inv_diag, prob.x, prob.rtol, prob.atol, prob.maxiter, user_stream);
}

}  // namespace msx
