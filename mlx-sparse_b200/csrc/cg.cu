// Plain CG and Jacobi-preconditioned CG on one GPU, with the whole Krylov loop
// on the device.
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

enum Kind { kCG = 0, kPCG = 1 };

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
// all partials into state->red. Returns true in thread 0 of the last CTA.
__device__ bool reduce_to_state(double (&v)[4], double *partials, CgState *st) {
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
    return true;
  }
  return false;
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
            int64_t n, double *partials, CgState *st, float rtol, float atol, bool decide) {
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
    } else {
      const float inv = inv_diag[i];
      const float zi = __fmul_rn(inv, ri);
      z[i] = zi;
      p[i] = zi;
      v[2] += (double)ri * (double)zi;
      if (!(finite_f(ri) && finite_f(zi) && finite_f(inv))) v[3] += 1.0;
    }
  }
  if (reduce_to_state(v, partials, st) && decide) decide_init(st, kind, rtol, atol);
}

// Fuses p.Ap, p.p, Ap.Ap (and the non-finite count) into the SpMV row
// epilogue; the last CTA makes the step decision.
struct DotsEpilogue {
  static constexpr int kMinBlocks = 6;  // room for the fp64 accumulators
  const float *p;
  double *partials;
  CgState *st;
  int kind;
  bool decide;
  double pap, pp, apap, bad;
  __device__ __forceinline__ bool skip() const { return st->status != kStatusRunning; }
  __device__ __forceinline__ void row(int64_t r, float apv) {
    const float pv = __ldg(p + r);
    pap += (double)pv * (double)apv;
    pp += (double)pv * (double)pv;
    apap += (double)apv * (double)apv;
    if (!(finite_f(pv) && finite_f(apv))) bad += 1.0;
  }
  __device__ __forceinline__ void finish() {
    double v[4] = {pap, pp, apap, bad};
    if (reduce_to_state(v, partials, st) && decide) decide_spmv(st, kind);
  }
};

__global__ void __launch_bounds__(kThreads)
dots_kernel(int kind, const float *__restrict__ p, const float *__restrict__ ap, int64_t n, double *partials,
            CgState *st, bool decide) {
  if (st->status != kStatusRunning) return;
  double v[4] = {0.0, 0.0, 0.0, 0.0};
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float pv = p[i], av = ap[i];
    v[0] += (double)pv * (double)av;
    v[1] += (double)pv * (double)pv;
    v[2] += (double)av * (double)av;
    if (!(finite_f(pv) && finite_f(av))) v[3] += 1.0;
  }
  if (reduce_to_state(v, partials, st) && decide) decide_spmv(st, kind);
}

__global__ void __launch_bounds__(kThreads)
update_kernel(int kind, float *__restrict__ x, float *__restrict__ r, float *__restrict__ z,
              const float *__restrict__ p, const float *__restrict__ ap, const float *__restrict__ inv_diag,
              int64_t n, double *partials, CgState *st, bool decide) {
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
  if (reduce_to_state(v, partials, st) && decide) decide_update(st, kind);
}

__global__ void __launch_bounds__(kThreads)
pupdate_kernel(int kind, const float *__restrict__ r, const float *__restrict__ z, float *__restrict__ p, int64_t n,
               double *partials, CgState *st, bool decide) {
  if (st->status != kStatusRunning) return;
  if (kind == kCG) {
    const double beta = st->beta_d;
    double v[4] = {0.0, 0.0, 0.0, 0.0};
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x) {
      const double pc = __dadd_rn((double)r[i], __dmul_rn(beta, (double)p[i]));
      const float pf = __double2float_rn(pc);
      if (!finite_d(pc) || !finite_f(pf)) {
        v[0] += 1.0;
        continue;
      }
      p[i] = pf;
    }
    if (reduce_to_state(v, partials, st) && decide) decide_pupdate(st);
  } else {
    const float beta = st->beta_f;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t first = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    int64_t done = 0;
    if (aligned16(z) && aligned16(p)) {
      const int64_t n4 = n / 4;
      for (int64_t i = first; i < n4; i += stride) {
        const float4 zv = __ldcs(reinterpret_cast<const float4 *>(z) + i);
        float4 pv = reinterpret_cast<const float4 *>(p)[i];
        pv.x = __fadd_rn(zv.x, __fmul_rn(beta, pv.x));
        pv.y = __fadd_rn(zv.y, __fmul_rn(beta, pv.y));
        pv.z = __fadd_rn(zv.z, __fmul_rn(beta, pv.z));
        pv.w = __fadd_rn(zv.w, __fmul_rn(beta, pv.w));
        reinterpret_cast<float4 *>(p)[i] = pv;
      }
      done = n4 * 4;
    }
    for (int64_t i = done + first; i < n; i += stride) p[i] = __fadd_rn(z[i], __fmul_rn(beta, p[i]));
  }
}

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

CgResult cg_solve(const CgProblem &prob, cudaStream_t user_stream) {
  const int kind = prob.inv_diag ? kPCG : kCG;
  const int64_t n = prob.n;
  const CgDist *dist = prob.dist;
  const bool decide = dist == nullptr;
#if !defined(MSX_HAVE_NCCL)
  if (dist) fail(MSX_ERR_RUNTIME, "this build has no NCCL: multi-GPU CG is unavailable.");
#endif
  // A private stream: graphs cannot be captured on the legacy default stream.
  cudaStream_t s;
  MSX_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
  struct StreamGuard {
    cudaStream_t s;
    ~StreamGuard() { cudaStreamDestroy(s); }
  } sguard{s};
  cudaEvent_t ev;
  MSX_CUDA(cudaEventCreateWithFlags(&ev, cudaEventDisableTiming));
  struct EventGuard {
    cudaEvent_t e;
    ~EventGuard() { cudaEventDestroy(e); }
  } eguard{ev};
  MSX_CUDA(cudaEventRecord(ev, user_stream));
  MSX_CUDA(cudaStreamWaitEvent(s, ev, 0));

  // Row-length bins of the matrix (built once per solve, in stream scratch).
  std::vector<std::unique_ptr<Scratch>> keep;
  BinnedPlan plan;
  build_binned_plan(prob.index_dtype, prob.indptr, n, prob.nnz, s,
                    [&](size_t bytes) -> void * {
                      keep.emplace_back(new Scratch(bytes, s));
                      return keep.back()->ptr;
                    },
                    plan);
  const bool fused = plan.n_long == 0;
  const int red_grid = elementwise_grid(n);
  int64_t spmv_grid_n = 0;
  dispatch_index(prob.index_dtype, [&](auto ityp) {
    using I = decltype(ityp);
    spmv_grid_n = std::max(binned_grid<float, I, DotsEpilogue>(plan), binned_grid<float, I, NoEpilogue>(plan));
  });
  const int64_t max_grid = std::max<int64_t>(red_grid, spmv_grid_n);

  // scratch layout
  const size_t vec = sizeof(float) * (size_t)std::max<int64_t>(n, 1);
  auto al = [](size_t b) { return (b + 255) & ~size_t(255); };
  size_t off = 0;
  const size_t o_state = off; off += al(sizeof(CgState));
  const size_t o_part = off;  off += al(sizeof(double) * 4 * max_grid);
  const size_t o_carry = off; off += al(sizeof(float) * std::max<int64_t>(plan.n_chunks, 1));
  const size_t o_r = off;     off += al(vec);
  const size_t o_z = off;     off += al(kind == kPCG ? vec : 0);
  const size_t o_p = off;     off += al(sizeof(float) * (size_t)std::max<int64_t>(prob.n_cols, 1));
  const size_t o_ap = off;    off += al(vec);
  int64_t n_send = 0;
  if (dist)
    for (int q = 0; q < dist->n_peers; ++q) n_send += dist->send_counts[q];
  const size_t o_send = off;  off += al(sizeof(float) * (size_t)std::max<int64_t>(n_send, 1));
  const size_t o_xh = off;    off += al(dist ? sizeof(float) * (size_t)std::max<int64_t>(prob.n_cols, 1) : 0);
  Scratch scratch(off, s);
  char *base = scratch.as<char>();
  CgState *st = reinterpret_cast<CgState *>(base + o_state);
  double *partials = reinterpret_cast<double *>(base + o_part);
  float *carry = reinterpret_cast<float *>(base + o_carry);
  float *r = reinterpret_cast<float *>(base + o_r);
  float *z = kind == kPCG ? reinterpret_cast<float *>(base + o_z) : nullptr;
  float *p = reinterpret_cast<float *>(base + o_p);
  float *ap = reinterpret_cast<float *>(base + o_ap);
  float *sendbuf = reinterpret_cast<float *>(base + o_send);
  float *xh = dist ? reinterpret_cast<float *>(base + o_xh) : nullptr;

  // Multi-GPU plumbing (all ranks issue the same sequence of collectives).
  auto exchange = [&](float *v, cudaStream_t q) {
#if defined(MSX_HAVE_NCCL)
    if (!dist) return;
    if (n_send > 0) {
      halo_pack_kernel<<<(unsigned)ceil_div(n_send, 256), 256, 0, q>>>(v, dist->send_idx, sendbuf, n_send);
      MSX_CHECK_LAUNCH();
    }
    ncclComm_t comm = static_cast<ncclComm_t>(dist->comm);
    auto nccl = [](ncclResult_t r) {
      if (r != ncclSuccess) fail(MSX_ERR_RUNTIME, std::string("NCCL: ") + ncclGetErrorString(r));
    };
    nccl(ncclGroupStart());
    int64_t so = 0, ro = 0;
    for (int k = 0; k < dist->n_peers; ++k) {
      if (dist->send_counts[k] > 0)
        nccl(ncclSend(sendbuf + so, (size_t)dist->send_counts[k], ncclFloat, dist->peers[k], comm, q));
      if (dist->recv_counts[k] > 0)
        nccl(ncclRecv(v + n + ro, (size_t)dist->recv_counts[k], ncclFloat, dist->peers[k], comm, q));
      so += dist->send_counts[k];
      ro += dist->recv_counts[k];
    }
    nccl(ncclGroupEnd());
#else
    (void)v;
    (void)q;
#endif
  };
  auto reduce_decide = [&](int which, cudaStream_t q) {
#if defined(MSX_HAVE_NCCL)
    if (!dist) return;
    ncclResult_t r = ncclAllReduce(st->red, st->red, 4, ncclDouble, ncclSum, static_cast<ncclComm_t>(dist->comm), q);
    if (r != ncclSuccess) fail(MSX_ERR_RUNTIME, std::string("NCCL: ") + ncclGetErrorString(r));
    decide_kernel<<<1, 1, 0, q>>>(st, which, kind, prob.rtol, prob.atol);
    MSX_CHECK_LAUNCH();
#else
    (void)which;
    (void)q;
#endif
  };

  CgState init{};
  init.status = kStatusRunning;
  init.it = 1;
  init.maxiter = prob.maxiter;
  MSX_CUDA(cudaMemcpyAsync(st, &init, sizeof(CgState), cudaMemcpyHostToDevice, s));
  MSX_CUDA(cudaMemcpyAsync(prob.x, prob.x0, sizeof(float) * n, cudaMemcpyDeviceToDevice, s));

  // r0 = b - A x0 (the halo of x0 comes from its owners first)
  const float *x_in = prob.x;
  if (dist) {
    MSX_CUDA(cudaMemcpyAsync(xh, prob.x0, sizeof(float) * n, cudaMemcpyDeviceToDevice, s));
    exchange(xh, s);
    x_in = xh;
  }
  spmv_binned_run(MSX_F32, prob.index_dtype, plan, prob.data, prob.indices, prob.indptr, x_in, ap, carry, s);
  init_kernel<<<red_grid, kThreads, 0, s>>>(kind, prob.b, prob.x, ap, prob.inv_diag, r, z, p, n, partials, st,
                                            prob.rtol, prob.atol, decide);
  MSX_CHECK_LAUNCH();
  reduce_decide(0, s);

  CgState host{};
  MSX_CUDA(cudaMemcpyAsync(&host, st, sizeof(CgState), cudaMemcpyDeviceToHost, s));
  MSX_CUDA(cudaStreamSynchronize(s));

  auto enqueue_iteration = [&](cudaStream_t q) {
    exchange(p, q);
    if (fused) {
      dispatch_index(prob.index_dtype, [&](auto ityp) {
        using I = decltype(ityp);
        DotsEpilogue epi{p, partials, st, kind, decide, 0.0, 0.0, 0.0, 0.0};
        launch_spmv_binned<float, I, DotsEpilogue>(plan, prob.data, static_cast<const I *>(prob.indices),
                                                   static_cast<const I *>(prob.indptr), p, ap, carry, epi, q);
      });
    } else {
      spmv_binned_run(MSX_F32, prob.index_dtype, plan, prob.data, prob.indices, prob.indptr, p, ap, carry, q);
      dots_kernel<<<red_grid, kThreads, 0, q>>>(kind, p, ap, n, partials, st, decide);
      MSX_CHECK_LAUNCH();
    }
    reduce_decide(1, q);
    update_kernel<<<red_grid, kThreads, 0, q>>>(kind, prob.x, r, z, p, ap, prob.inv_diag, n, partials, st, decide);
    MSX_CHECK_LAUNCH();
    reduce_decide(2, q);
    pupdate_kernel<<<red_grid, kThreads, 0, q>>>(kind, r, z, p, n, partials, st, decide);
    MSX_CHECK_LAUNCH();
    if (kind == kCG) reduce_decide(3, q);
  };

  if (host.status == kStatusRunning) {
    // Iterations per graph launch: about a millisecond of work per batch.
    const double bytes_per_iter = 8.0 * prob.nnz + 56.0 * n;
    int batch = (int)std::max(1.0, std::min(64.0, 5.0e9 * 1e-3 / std::max(bytes_per_iter, 1.0)));
    batch = std::max(4, batch);
    batch = std::min(batch, std::max(prob.maxiter, 1));
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    MSX_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    try {
      for (int k = 0; k < batch; ++k) enqueue_iteration(s);
    } catch (...) {
      cudaStreamEndCapture(s, &graph);
      if (graph) cudaGraphDestroy(graph);
      throw;
    }
    MSX_CUDA(cudaStreamEndCapture(s, &graph));
    struct GraphGuard {
      cudaGraph_t g;
      cudaGraphExec_t e;
      ~GraphGuard() {
        if (e) cudaGraphExecDestroy(e);
        if (g) cudaGraphDestroy(g);
      }
    } gguard{graph, nullptr};
    MSX_CUDA(cudaGraphInstantiate(&exec, graph, 0));
    gguard.e = exec;
    int *status_host = nullptr;
    MSX_CUDA(cudaMallocHost(&status_host, sizeof(int)));
    struct HostGuard {
      int *p;
      ~HostGuard() { cudaFreeHost(p); }
    } hguard{status_host};
    int64_t launched = 0;
    while (true) {
      MSX_CUDA(cudaGraphLaunch(exec, s));
      launched += batch;
      MSX_CUDA(cudaMemcpyAsync(status_host, &st->status, sizeof(int), cudaMemcpyDeviceToHost, s));
      MSX_CUDA(cudaStreamSynchronize(s));
      if (*status_host != kStatusRunning || launched >= prob.maxiter) break;
    }
    MSX_CUDA(cudaMemcpyAsync(&host, st, sizeof(CgState), cudaMemcpyDeviceToHost, s));
    MSX_CUDA(cudaStreamSynchronize(s));
  }

  CgResult res{};
  res.info = host.status;
  res.iterations = host.completed;
  if (kind == kCG) {
    res.residual = (float)std::sqrt(std::max(host.rr, 0.0));
  } else {
    res.residual = std::sqrt(std::max(host.true_rr, 0.0f));
  }
  if (host.status == kStatusRunning) fail(MSX_ERR_RUNTIME, "CG solve ended without a status (internal error).");
  // order the caller's stream after the solve
  MSX_CUDA(cudaEventRecord(ev, s));
  MSX_CUDA(cudaStreamWaitEvent(user_stream, ev, 0));
  return res;
}

}  // namespace msx
