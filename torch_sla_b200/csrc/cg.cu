// Jacobi-preconditioned CG (and plain CG when dinv == NULL) with the
// stopping rule of pcg_solve_optimized (backends/pytorch_backend.py:1262-1362):
// at the start of iteration i stop if (r,r) < max(atol, rtol*||b||)^2 and
// report i iterations.
//
// Streamed path (large systems), per iteration:
//   K_P  p_new = p_old*beta + M^{-1} r             (streaming pass)
//   K_A  Ap = A p_new, partial (p_new, Ap)
//        last block: alpha = (r,z) / (p,Ap)
//   K_B  x += alpha p ; r -= alpha Ap ; partial (r,r), (r, M^{-1} r)
//        last block: beta, convergence / maxiter bookkeeping
// (or, with SLA_CG_SPLIT 0, K_P fused into K_A's gather). HBM per
// iteration: matrix + 12 vector passes on average (r, dinv, p_old read and
// p_new written by K_P; p_new read and Ap written by K_A; r, Ap, dinv read
// and r written by K_B, plus x, p, p_prev read and x written at every
// other iteration).
// The scalar recurrences stay on the device; the host polls a pinned flag
// once per chunk of iterations with one chunk in flight.
//
// Persistent path (small systems, vectors L2-resident): the same two phases
// in one cooperative launch separated by a bounded grid barrier.

#include <cooperative_groups.h>

#include <type_traits>

#include "solver.cuh"

namespace sla {

struct CgState {
  double rz;
  double rr;
  double pAp;
  double alpha;
  double alpha_prev;  // alpha of the previous (even) iteration, whose x update is pending
  double beta;
  double tol_sq;
  long long iter;
  long long maxiter;
  long long iters_out;
  int done;  // 0 running, 1 converged, 2 maxiter, 3 non-finite, 4 timeout
  int pad;
  unsigned counter[4];
  GridBarrier bar;
};

enum { kRunning = 0, kConverged = 1, kMaxiter = 2, kNonFinite = 3, kTimeout = 4 };

// Threads per block of the persistent kernel: its two grid barriers per
// iteration cost more with more blocks, so it runs fewer, larger blocks
// than the streamed kernels.
#ifndef SLA_PERSIST_BLOCK
#define SLA_PERSIST_BLOCK 256
#endif
constexpr int kPBlock = SLA_PERSIST_BLOCK;
constexpr int kPWarps = kPBlock / 32;

// Every block of the persistent kernel sums the NV x gridDim partials in the
// same order.
template <int NV>
__device__ __forceinline__ void reduce_partials(double (&v)[NV], const double *parts,
                                                double *smem) {
  const unsigned G = gridDim.x;
#pragma unroll
  for (int k = 0; k < NV; ++k) v[k] = 0.0;
  for (unsigned i = threadIdx.x; i < G; i += kPBlock) {
#pragma unroll
    for (int k = 0; k < NV; ++k) v[k] += ld_l2(parts + k * G + i);
  }
  block_sum<NV, kPBlock>(v, smem);
}

template <typename T, bool PREC, bool COH>
struct CgPGather {
  const T *r;
  const T *dinv;
  const T *p_old;
  T beta;
  __device__ __forceinline__ T operator()(int32_t c) const {
    T rc = COH ? ld_l2(r + c) : __ldg(r + c);
    T pc = COH ? ld_l2(p_old + c) : __ldg(p_old + c);
    T z = PREC ? mul_rn(__ldg(dinv + c), rc) : rc;
    return add_rn(mul_rn(pc, beta), z);
  }
};

template <typename T, bool PREC>
__global__ void __launch_bounds__(kBlock)
cg_init_kernel(int64_t n, const T *__restrict__ b, T *__restrict__ x, const T *__restrict__ Ax,
               const T *__restrict__ dinv, T *__restrict__ r, T *__restrict__ p_old, CgState *st,
               double *partials, double atol, double rtol) {
  __shared__ double smem[3 * kWarps];
  double acc[3] = {0.0, 0.0, 0.0};
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) {
    T bi = b[i];
    T ri = Ax ? sub_rn(bi, Ax[i]) : bi;
    if (!Ax) x[i] = T(0);
    r[i] = ri;
    p_old[i] = T(0);
    T zi = PREC ? mul_rn(dinv[i], ri) : ri;
    acc[0] += (double)ri * (double)ri;
    acc[1] += (double)ri * (double)zi;
    acc[2] += (double)bi * (double)bi;
  }
  if (last_block_sum<3, kBlock>(acc, partials, &st->counter[0], smem) && threadIdx.x == 0) {
    st->rr = acc[0];
    st->rz = acc[1];
    double tol = fmax(atol, rtol * sqrt(acc[2]));
    st->tol_sq = tol * tol;
    st->beta = 0.0;
    st->iter = 0;
    if (acc[0] < st->tol_sq) { st->done = kConverged; st->iters_out = 0; }
    else if (st->maxiter <= 0) { st->done = kMaxiter; st->iters_out = 0; }
    else if (!isfinite(acc[0])) { st->done = kNonFinite; st->iters_out = st->maxiter; }
    else st->done = kRunning;
  }
}

template <typename T, bool PREC, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
cg_spmv_kernel(Sell<T> A, const T *__restrict__ r, const T *__restrict__ dinv,
               const T *__restrict__ p_old, T *__restrict__ p_new, T *__restrict__ Ap, CgState *st,
               double *partials) {
  __shared__ double smem[kWarps];
  if (*(volatile int *)&st->done) return;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  CgPGather<T, PREC, false> g{r, dinv, p_old, (T)st->beta};
  double acc[1] = {0.0};
  for_each_slice<WS>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
    T sum = sell_row_at<WS>(A, s, sbase, swidth, lane, g);
    const int64_t slot = s * 32 + lane;
    if (slot < A.n_slots) {
      const int64_t row = slot_row(A, slot);
      T pn = g((int32_t)row);
      p_new[row] = pn;
      Ap[row] = sum;
      acc[0] += (double)pn * (double)sum;
    }
  });
  if (last_block_sum<1, kBlock>(acc, partials, &st->counter[1], smem) && threadIdx.x == 0) {
    st->pAp = acc[0];
    st->alpha = st->rz / acc[0];
  }
}

// 16-byte vector of a streaming pass: two doubles or four floats.
template <typename T> struct Vec16;
template <> struct Vec16<double> { using type = double2; static constexpr int E = 2; };
template <> struct Vec16<float> { using type = float4; static constexpr int E = 4; };
template <typename T, typename V>
__device__ __forceinline__ T &lane_of(V &v, int u) { return reinterpret_cast<T *>(&v)[u]; }

// Split K_A (kCgSplit): p_new = p_old*beta + M^{-1} r is formed once per row
// by cg_pform_kernel (a streaming pass) and K_A is a plain SpMV over p_new
// with the L2 prefetch of the next slice's values; same arithmetic, same
// row sums and dot order as the fused K_A, which forms p inside the gather,
// once per entry.

template <typename T, bool PREC, bool VEC>
__global__ void __launch_bounds__(kBlock)
cg_pform_kernel(int64_t n, const T *__restrict__ r, const T *__restrict__ dinv,
                const T *__restrict__ p_old, T *__restrict__ p_new, const CgState *st) {
  if (*(volatile const int *)&st->done) return;
  const T beta = (T)st->beta;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  auto pf = [&](T pc, T rc, T dc) { return add_rn(mul_rn(pc, beta), PREC ? mul_rn(dc, rc) : rc); };
  int64_t tail = 0;
  if (VEC) {
    using V = typename Vec16<T>::type;
    constexpr int E = Vec16<T>::E;
    const int64_t nv = n / E;
    for (int64_t i = tid; i < nv; i += stride) {
      V rv = __ldcs((const V *)r + i), pv = __ldcs((const V *)p_old + i);
      V dv = rv;
      if (PREC) dv = __ldg((const V *)dinv + i);
      V out;
#pragma unroll
      for (int u = 0; u < E; ++u)
        lane_of<T>(out, u) = pf(lane_of<T>(pv, u), lane_of<T>(rv, u), lane_of<T>(dv, u));
      ((V *)p_new)[i] = out;
    }
    tail = nv * E;
  }
  for (int64_t i = tail + tid; i < n; i += stride)
    p_new[i] = pf(p_old[i], r[i], PREC ? dinv[i] : T(0));
}

template <typename T, int WS>
__global__ void __launch_bounds__(kBlock, kSpmvMinBlocks)
cg_spmv_split_kernel(Sell<T> A, const T *__restrict__ p, T *__restrict__ Ap, CgState *st,
                     double *partials) {
  __shared__ double smem[kWarps];
  if (*(volatile int *)&st->done) return;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  PlainGather<T> g{p};
  double acc[1] = {0.0};
  if constexpr (std::is_same_v<T, float> && kSolverRowsX2<WS>) {
    // float32 7-wide views: two rows per lane (p 8-byte aligned: checked
    // by the launch)
    for_each_slice_x2(A.n_slices, warp, nwarps, lane, [&](int64_t s, int hl) {
      int64_t r0, r1;
      float s0, s1;
      sell_rows_x2<WS>(A, s, hl, p, r0, r1, s0, s1);
      if (r0 >= 0) {
        Ap[r0] = s0;
        acc[0] += (double)__ldg(p + r0) * (double)s0;
      }
      if (r1 >= 0) {
        Ap[r1] = s1;
        acc[0] += (double)__ldg(p + r1) * (double)s1;
      }
    });
  } else {
    for_each_slice<WS, true>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
      T sum = sell_row_at<WS>(A, s, sbase, swidth, lane, g);
      const int64_t slot = s * 32 + lane;
      if (slot < A.n_slots) {
        const int64_t row = slot_row(A, slot);
        const T pn = __ldg(p + row);
        Ap[row] = sum;
        acc[0] += (double)pn * (double)sum;
      }
    });
  }
  if (last_block_sum<1, kBlock>(acc, partials, &st->counter[1], smem) && threadIdx.x == 0) {
    st->pAp = acc[0];
    st->alpha = st->rz / acc[0];
  }
}

// K_A of one iteration, fused or split.
template <typename T, bool PREC, int WS>
struct KaLaunch {
  int grid = 0, grid_p = 0;
  bool vec = false;
  void init(int64_t n, const void *r, const void *dinv, const void *pA, const void *pB) {
    if (kCgSplit) {
      grid = spmv_grid();
      grid_p = occupancy_grid((const void *)cg_pform_kernel<T, PREC, true>);
      vec = aligned16(r, pA, pB) && (!PREC || aligned16(dinv));
    } else {
      grid = occupancy_grid((const void *)cg_spmv_kernel<T, PREC, WS>);
    }
  }
  // prof: time the launches with the sampling profiler (class 0 the SpMV,
  // class 2 the p-forming pass).
  int run(int64_t it, bool prof, const Sell<T> &A, const T *r, const T *dinv, const T *p_old,
          T *p_new, T *Ap, CgState *st, double *part, cudaStream_t s) const {
    cudaEvent_t ev;
    if (kCgSplit) {
      const int64_t n = A.n_slots;
      if (prof) profiler().begin(2, it, s, &ev);
      if (vec)
        SLA_LAUNCH((cg_pform_kernel<T, PREC, true>), grid_p, kBlock, 0, s, n, r, dinv, p_old, p_new, st);
      else
        SLA_LAUNCH((cg_pform_kernel<T, PREC, false>), grid_p, kBlock, 0, s, n, r, dinv, p_old, p_new, st);
      if (prof) profiler().end(2, s, ev);
      if (prof) profiler().begin(0, it, s, &ev);
      SLA_LAUNCH((cg_spmv_split_kernel<T, WS>), grid, kBlock, 0, s, A, (const T *)p_new, Ap, st, part);
      if (prof) profiler().end(0, s, ev);
    } else {
      if (prof) profiler().begin(0, it, s, &ev);
      SLA_LAUNCH((cg_spmv_kernel<T, PREC, WS>), grid, kBlock, 0, s, A, r, dinv, p_old, p_new, Ap,
                 st, part);
      if (prof) profiler().end(0, s, ev);
    }
    return SLA_OK;
  }
};

// r -= alpha Ap (torch addcmul_ rounding) and the two dots.
template <typename T, bool PREC>
__device__ __forceinline__ void cg_rupd(T &ri, T api, T di, T alpha, double (&acc)[2]) {
  ri = sub_rn(ri, mul_rn(alpha, api));
  T zi = PREC ? mul_rn(di, ri) : ri;
  acc[0] += (double)ri * (double)ri;
  acc[1] += (double)ri * (double)zi;
}

// x updates are applied two iterations at a time: at an even iteration the
// kernel only updates r; at the following odd one it applies
// x = (x + alpha_prev p_prev) + alpha p -- the same two roundings as two
// separate x += alpha p steps, so x is bitwise unchanged -- while both
// search directions still sit in the ping-pong buffers. That saves the x
// read, the x write and the p read of every other iteration. A solve that
// stops after an even iteration gets the pending step from cg_xflush_kernel.
template <typename T, bool PREC, bool VEC, bool XU>
__global__ void __launch_bounds__(kBlock)
cg_update_kernel(int64_t n, T *__restrict__ x, T *__restrict__ r, const T *__restrict__ p,
                 const T *__restrict__ p_prev, const T *__restrict__ Ap,
                 const T *__restrict__ dinv, CgState *st, double *partials) {
  __shared__ double smem[2 * kWarps];
  if (*(volatile int *)&st->done) return;
  const T alpha = (T)st->alpha;
  const T alpha_prev = (T)st->alpha_prev;
  double acc[2] = {0.0, 0.0};
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  auto xstep = [&](T xi, T pp, T pc) {
    return add_rn(add_rn(xi, mul_rn(alpha_prev, pp)), mul_rn(alpha, pc));
  };
  if (VEC) {
    using V = typename Vec16<T>::type;
    constexpr int E = Vec16<T>::E;
    const int64_t nv = n / E;
    for (int64_t i = tid; i < nv; i += stride) {
      V rv = ((V *)r)[i];
      V av = __ldcs((const V *)Ap + i);
      V dv = av;
      if (PREC) dv = __ldg((const V *)dinv + i);
      if (XU) {
        V xv = ((V *)x)[i];
        V pv = __ldcs((const V *)p + i), qv = __ldcs((const V *)p_prev + i);
#pragma unroll
        for (int u = 0; u < E; ++u)
          lane_of<T>(xv, u) = xstep(lane_of<T>(xv, u), lane_of<T>(qv, u), lane_of<T>(pv, u));
        ((V *)x)[i] = xv;
      }
#pragma unroll
      for (int u = 0; u < E; ++u)
        cg_rupd<T, PREC>(lane_of<T>(rv, u), lane_of<T>(av, u), lane_of<T>(dv, u), alpha, acc);
      ((V *)r)[i] = rv;
    }
    for (int64_t i = nv * E + tid; i < n; i += stride) {
      if (XU) x[i] = xstep(x[i], p_prev[i], p[i]);
      T ri = r[i];
      cg_rupd<T, PREC>(ri, Ap[i], PREC ? dinv[i] : T(0), alpha, acc);
      r[i] = ri;
    }
  } else {
    for (int64_t i = tid; i < n; i += stride) {
      if (XU) x[i] = xstep(x[i], p_prev[i], p[i]);
      T ri = r[i];
      cg_rupd<T, PREC>(ri, Ap[i], PREC ? dinv[i] : T(0), alpha, acc);
      r[i] = ri;
    }
  }
  if (last_block_sum<2, kBlock>(acc, partials, &st->counter[2], smem) && threadIdx.x == 0) {
    const long long it = st->iter + 1;
    st->iter = it;
    st->alpha_prev = st->alpha;
    st->rr = acc[0];
    st->beta = acc[1] / st->rz;
    st->rz = acc[1];
    if (acc[0] < st->tol_sq) { st->done = kConverged; st->iters_out = it; }
    else if (!isfinite(acc[0])) { st->done = kNonFinite; st->iters_out = st->maxiter; }
    else if (it >= st->maxiter) { st->done = kMaxiter; st->iters_out = st->maxiter; }
  }
}

// The x step of a last even iteration (st->iter odd), left pending by the
// deferred update; p_last is that iteration's search direction.
template <typename T>
__global__ void __launch_bounds__(kBlock)
cg_xflush_kernel(int64_t n, T *__restrict__ x, const T *__restrict__ p_last, const CgState *st) {
  if ((st->iter & 1) == 0 || st->done == kTimeout) return;
  const T alpha = (T)st->alpha_prev;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (; i < n; i += stride) x[i] = add_rn(x[i], mul_rn(alpha, p_last[i]));
}

template <typename T, bool PREC, int WS>
__global__ void __launch_bounds__(kPBlock, 1024 / kPBlock)
cg_persistent_kernel(Sell<T> A, int64_t n, T *__restrict__ x, T *__restrict__ r,
                     const T *__restrict__ dinv, T *pA, T *pB, T *__restrict__ Ap, CgState *st,
                     double *partA, double *partB) {
  __shared__ double smem[2 * kPWarps];
  if (*(volatile int *)&st->done) return;
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  double rz = st->rz, rr = st->rr;
  const double tol_sq = st->tol_sq;
  const long long maxiter = st->maxiter;
  double beta = 0.0;
  T *p_old = pA, *p_new = pB;
  int done = kMaxiter;
  long long iters = maxiter;
  for (long long k = 0; k < maxiter; ++k) {
    // phase A: p_new = p_old*beta + M^{-1} r (fused into the gather), Ap = A p_new
    CgPGather<T, PREC, true> g{r, dinv, p_old, (T)beta};
    double a1[1] = {0.0};
    for_each_slice<WS>(A, warp, nwarps, lane, [&](int64_t s, int32_t sbase, int swidth) {
      T sum = sell_row_at<WS>(A, s, sbase, swidth, lane, g);
      const int64_t slot = s * 32 + lane;
      if (slot < n) {
        const int64_t row = slot_row(A, slot);
        T pn = g((int32_t)row);
        p_new[row] = pn;
        Ap[row] = sum;
        a1[0] += (double)pn * (double)sum;
      }
    });
    block_sum<1, kPBlock>(a1, smem);
    if (threadIdx.x == 0) partA[blockIdx.x] = a1[0];
    if (!grid_sync(&st->bar)) { done = kTimeout; break; }
    reduce_partials<1>(a1, partA, smem);
    const T alpha = (T)(rz / a1[0]);
    // phase B: x, r update and the two residual dots
    double a2[2] = {0.0, 0.0};
    for (int64_t i = tid; i < n; i += nthreads) {
      T xi = add_rn(x[i], mul_rn(alpha, ld_l2(p_new + i)));
      T ri = sub_rn(r[i], mul_rn(alpha, ld_l2(Ap + i)));
      x[i] = xi;
      r[i] = ri;
      T zi = PREC ? mul_rn(dinv[i], ri) : ri;
      a2[0] += (double)ri * (double)ri;
      a2[1] += (double)ri * (double)zi;
    }
    block_sum<2, kPBlock>(a2, smem);
    if (threadIdx.x == 0) { partB[blockIdx.x] = a2[0]; partB[gridDim.x + blockIdx.x] = a2[1]; }
    if (!grid_sync(&st->bar)) { done = kTimeout; break; }
    reduce_partials<2>(a2, partB, smem);
    rr = a2[0];
    beta = a2[1] / rz;
    rz = a2[1];
    if (rr < tol_sq) { done = kConverged; iters = k + 1; break; }
    if (!isfinite(rr)) { done = kNonFinite; iters = maxiter; break; }
    T *t = p_old; p_old = p_new; p_new = t;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    st->rr = rr;
    st->rz = rz;
    st->done = done;
    st->iters_out = iters;
  }
}

// ------------------------------------------------- thread-block cluster CG
// Small stencil systems run inside ONE thread-block cluster (16 CTAs of 1024
// threads where the GPU allows that cluster size, else 8): CTA c owns R
// consecutive rows (R a multiple of 32, at most 4 per thread) and keeps
// their matrix values (diagonal-offset view), their search direction and
// their Jacobi inverse in shared memory, x and r in registers. The SpMV reads
// the search direction of rows owned by other CTAs through distributed
// shared memory, and the three synchronisation points of an iteration
// (search direction published; (p, Ap) partials; (r, r) and (r, z) partials)
// are hardware cluster barriers rather than grid barriers through global
// memory. Partial sums go through warp butterflies in a fixed order, each
// CTA pushes its total into every CTA's shared memory before the barrier,
// and every warp then sums the per-CTA totals the same way, so all CTAs
// take the same decisions with one CTA barrier per reduction. Same recurrences and roundings as the streamed
// path (x updated every iteration: the same roundings as its deferred
// two-step update).
constexpr int kClThreads = 1024;
constexpr int kClRowsPerThread = 4;
constexpr int kClRowsMax = kClThreads * kClRowsPerThread;

constexpr int kClMaxCtas = 16;

// Sum over a warp in a fixed butterfly order: every lane gets the same total.
__device__ __forceinline__ double warp_total(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
  return v;
}

// Cluster-wide total of NV doubles per thread, identical in every thread of
// every CTA: warp butterflies, the 32 warp totals summed by warp 0 the same
// way, the CTA total stored into slot `me` of every CTA's `tot` (DSMEM), one
// cluster barrier, then every warp sums the ncta slots with a butterfly.
// wsm: NV x 32 doubles of this CTA. One CTA barrier and one cluster barrier.
template <int NV>
__device__ __forceinline__ void cluster_total(double (&v)[NV], double *wsm, double *tot,
                                              cooperative_groups::cluster_group &cl,
                                              unsigned me, unsigned ncta) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const double w = warp_total(v[k]);
    if (lane == 0) wsm[k * 32 + warp] = w;
  }
  __syncthreads();
  if (warp == 0) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const double t = warp_total(wsm[k * 32 + lane]);
      if (lane < (int)ncta) cl.map_shared_rank(tot, lane)[k * kClMaxCtas + me] = t;
    }
  }
  cl.sync();
#pragma unroll
  for (int k = 0; k < NV; ++k)
    v[k] = warp_total(lane < (int)ncta ? tot[k * kClMaxCtas + lane] : 0.0);
}

template <typename T, bool PREC, int W>
__global__ void __launch_bounds__(kClThreads, 1)
cg_cluster_kernel(Sell<T> A, int64_t n, int32_t R, T *__restrict__ x, const T *__restrict__ r_in,
                  const T *__restrict__ dinv, CgState *st) {
  namespace cgx = cooperative_groups;
  cgx::cluster_group cl = cgx::this_cluster();
  extern __shared__ __align__(16) unsigned char cl_smem[];
  T *sv = reinterpret_cast<T *>(cl_smem);                  // [R * W] values
  T *sp = sv + (size_t)R * W;                               // [R] search direction
  T *sd = sp + R;                                           // [R] Jacobi inverse (PREC)
  double *tot_a = reinterpret_cast<double *>(sd + (PREC ? R : 0));  // [kClMaxCtas] (p,Ap)
  double *tot_b = tot_a + kClMaxCtas;                       // [2][kClMaxCtas] (r,r), (r,z)
  double *wsm_a = tot_b + 2 * kClMaxCtas;                   // [32] warp totals, (p,Ap)
  double *wsm_b = wsm_a + 32;                               // [2][32] warp totals, (r,r), (r,z)
  const int tid = threadIdx.x;
  const unsigned me = cl.block_rank();
  const unsigned ncta = cl.num_blocks();
  const int32_t n32 = (int32_t)n;
  const int32_t r0 = (int32_t)me * R;
  const int64_t vend = A.n_slices * 32 * W;
  for (int64_t i = tid; i < (int64_t)R * W; i += kClThreads)
    sv[i] = ((int64_t)r0 * W + i < vend) ? A.val[(int64_t)r0 * W + i] : T(0);
  if (PREC)
    for (int i = tid; i < R; i += kClThreads) sd[i] = (r0 + i < n32) ? dinv[r0 + i] : T(0);
  // slots of rows past n are never written by the loop, but a row near n
  // reaches them through the local branch of the gather (a column >= n
  // inside this CTA's range, with value 0): they must hold 0, not whatever
  // an earlier kernel left in shared memory (0 * NaN would be NaN)
  for (int i = tid; i < R; i += kClThreads) sp[i] = T(0);
  int32_t off[W];
#pragma unroll
  for (int j = 0; j < W; ++j) off[j] = A.off[j];
  const int32_t ncols = (int32_t)A.n_cols;
  T xr[kClRowsPerThread], rv[kClRowsPerThread], ap[kClRowsPerThread], pv[kClRowsPerThread];
  bool own[kClRowsPerThread];
#pragma unroll
  for (int q = 0; q < kClRowsPerThread; ++q) {
    const int lr = tid + q * kClThreads;
    own[q] = lr < R && r0 + lr < n32;
    xr[q] = own[q] ? x[r0 + lr] : T(0);
    rv[q] = own[q] ? r_in[r0 + lr] : T(0);
    pv[q] = T(0);
    ap[q] = T(0);
  }
  double rz = st->rz, rr = st->rr;
  const double tol_sq = st->tol_sq;
  const long long maxiter = st->maxiter;
  int done = st->done;
  long long iters = done == kRunning ? maxiter : st->iters_out;
  double beta = 0.0;
  __syncthreads();
  for (long long k = 0; done == kRunning && k < maxiter; ++k) {
    // 1: p = M^{-1} r + beta p, published to the cluster
#pragma unroll
    for (int q = 0; q < kClRowsPerThread; ++q) {
      if (own[q]) {
        const int lr = tid + q * kClThreads;
        const T z = PREC ? mul_rn(sd[lr], rv[q]) : rv[q];
        pv[q] = add_rn(mul_rn(pv[q], (T)beta), z);
        sp[lr] = pv[q];
      }
    }
    cl.sync();
    // 2: Ap (ascending diagonals, one FMA chain per row as in the streamed
    // path; columns owned by another CTA over DSMEM) and (p, Ap)
    double a1[1] = {0.0};
#pragma unroll
    for (int q = 0; q < kClRowsPerThread; ++q) {
      if (own[q]) {
        const int lr = tid + q * kClThreads;
        const int32_t row = r0 + lr;
        const T *vp = sv + (lr >> 5) * 32 * W + (lr & 31);
        T sum = T(0);
#pragma unroll
        for (int j = 0; j < W; ++j) {
          const int32_t c = row + off[j];
          const int32_t lc = c - r0;
          T pc = T(0);
          if ((uint32_t)lc < (uint32_t)R) {
            pc = sp[lc];
          } else if ((uint32_t)c < (uint32_t)ncols) {
            const int32_t owner = c / R;
            pc = cl.map_shared_rank(sp, owner)[c - owner * R];
          }
          sum = fma(vp[32 * j], pc, sum);
        }
        ap[q] = sum;
        a1[0] += (double)pv[q] * (double)sum;
      }
    }
    cluster_total<1>(a1, wsm_a, tot_a, cl, me, ncta);
    const T alpha = (T)(rz / a1[0]);
    // 3: x, r update and the two residual dots
    double a2[2] = {0.0, 0.0};
#pragma unroll
    for (int q = 0; q < kClRowsPerThread; ++q) {
      if (own[q]) {
        const int lr = tid + q * kClThreads;
        xr[q] = add_rn(xr[q], mul_rn(alpha, pv[q]));
        rv[q] = sub_rn(rv[q], mul_rn(alpha, ap[q]));
        const T z = PREC ? mul_rn(sd[lr], rv[q]) : rv[q];
        a2[0] += (double)rv[q] * (double)rv[q];
        a2[1] += (double)rv[q] * (double)z;
      }
    }
    cluster_total<2>(a2, wsm_b, tot_b, cl, me, ncta);
    rr = a2[0];
    beta = a2[1] / rz;
    rz = a2[1];
    const long long it = k + 1;
    if (rr < tol_sq) { done = kConverged; iters = it; }
    else if (!isfinite(rr)) { done = kNonFinite; iters = maxiter; }
    else if (it >= maxiter) { done = kMaxiter; iters = maxiter; }
  }
#pragma unroll
  for (int q = 0; q < kClRowsPerThread; ++q)
    if (own[q]) x[r0 + tid + q * kClThreads] = xr[q];
  if (me == 0 && tid == 0) {
    st->rr = rr;
    st->rz = rz;
    st->done = done;
    st->iters_out = iters;
    st->iter = 0;  // x is complete: no pending deferred step
  }
  cl.sync();  // no CTA leaves while another may still read its shared memory
}

// K_B of iteration `it`: x is updated at odd iterations only (see
// cg_update_kernel); p_new / p_old are that iteration's directions.
template <typename T, bool PREC>
static int update_launch(bool vec, int64_t it, int64_t n, T *x, T *r, const T *p_new,
                         const T *p_old, const T *Ap, const T *dinv, CgState *st, double *part,
                         cudaStream_t s) {
  auto go = [&](auto fn) -> int {
    SLA_LAUNCH(fn, occupancy_grid((const void *)fn), kBlock, 0, s, n, x, r, p_new, p_old, Ap, dinv,
               st, part);
    return SLA_OK;
  };
  const bool odd = (it & 1) != 0;
  if (vec) return odd ? go(cg_update_kernel<T, PREC, true, true>) : go(cg_update_kernel<T, PREC, true, false>);
  return odd ? go(cg_update_kernel<T, PREC, false, true>) : go(cg_update_kernel<T, PREC, false, false>);
}

// Launch of cg_cluster_kernel when the system fits one cluster: a
// diagonal-offset view (columns computed, values only in shared memory) with
// at most kClRowsMax rows per CTA and the CTA's values, search direction and
// Jacobi inverse within the shared-memory limit. *launched tells the caller
// whether it ran (false: use another path).
template <typename T, bool PREC, int WS>
static int cluster_launch(const Sell<T> &A, int64_t n, T *x, T *r, const T *dinv, CgState *st,
                          cudaStream_t s, bool *launched) {
  *launched = false;
  if constexpr (WS <= kDiagSpec) {
    return SLA_OK;
  } else {
    constexpr int W = WS - kDiagSpec;
    auto kern = cg_cluster_kernel<T, PREC, W>;
    int dev = 0, max_smem = 0;
    SLA_CUDA_TRY(cudaGetDevice(&dev));
    SLA_CUDA_TRY(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    for (int cl : {kClMaxCtas, 8}) {
      const int64_t R = (n + (int64_t)cl * 32 - 1) / ((int64_t)cl * 32) * 32;
      if (R > kClRowsMax) return SLA_OK;  // a smaller cluster only holds fewer rows
      const size_t smem = (size_t)R * W * sizeof(T) + (size_t)R * sizeof(T) * (PREC ? 2 : 1) +
                          (3 * kClMaxCtas + 3 * 32) * sizeof(double);
      if (smem > (size_t)max_smem) return SLA_OK;
      SLA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem));
      if (cl > 8)
        SLA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(cl);
      cfg.blockDim = dim3(kClThreads);
      cfg.dynamicSmemBytes = smem;
      cfg.stream = s;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = cl;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      cfg.attrs = at;
      cfg.numAttrs = 1;
      int fits = 0;
      if (cudaOccupancyMaxActiveClusters(&fits, kern, &cfg) != cudaSuccess || fits < 1) {
        cudaGetLastError();  // this cluster size is refused here: try the next
        continue;
      }
      const int32_t R32 = (int32_t)R;
      SLA_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, A, n, R32, x, (const T *)r, dinv, st));
      g_launches.fetch_add(1, std::memory_order_relaxed);
      *launched = true;
      return SLA_OK;
    }
    return SLA_OK;
  }
}

static size_t cg_ws_bytes(size_t elem, int64_t n) {
  size_t G = (size_t)solver_grid();
  return 4 * align_up(elem * (size_t)n) + 2 * align_up(4 * G * sizeof(double)) +
         align_up(sizeof(CgState));
}

template <typename T>
int spmv_launch(const sla_sell_t *A, const void *x, void *y, cudaStream_t s);

template <typename T, bool PREC, int WS>
static int pcg_impl(const sla_sell_t *Ad, const T *dinv, const T *b, T *x, bool guess,
                    double atol, double rtol, int64_t maxiter, int flags, void *ws,
                    size_t ws_bytes, sla_solve_info_t *info, cudaStream_t s) {
  Sell<T> A = make_sell<T>(Ad);
  const int64_t n = A.n_slots;
  Carver c(ws, ws_bytes);
  T *r = c.take<T>(n), *pA = c.take<T>(n), *pB = c.take<T>(n), *Ap = c.take<T>(n);
  const int G = solver_grid();
  double *part0 = c.take<double>(4 * (size_t)G), *part1 = c.take<double>(4 * (size_t)G);
  CgState *st = c.take<CgState>(1);
  if (!c.ok) return SLA_ERR_WORKSPACE;
  CgState init{};
  init.maxiter = maxiter;
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(CgState), cudaMemcpyHostToDevice, s));
  if (guess) SLA_TRY(spmv_launch<T>(Ad, x, Ap, s));
  SLA_LAUNCH((cg_init_kernel<T, PREC>), grid_for(n), kBlock, 0, s, n, b, x, guess ? Ap : nullptr,
             dinv, r, pA, st, part0, atol, rtol);

  const DeviceInfo &dev = device_info();
  bool persistent = false;
  int coop_grid = 0;
  if (flags != SLA_PCG_STREAMED && dev.coop) {
    int per_sm = 0;
    SLA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &per_sm, cg_persistent_kernel<T, PREC, WS>, kPBlock, 0));
    int want = (int)((n + kPBlock - 1) / kPBlock);
    int cap = per_sm * dev.sm_count;
    coop_grid = want < cap ? want : cap;
    if (coop_grid < 1) coop_grid = 1;
    bool small = n <= (int64_t)(1 << 20);
    persistent = per_sm > 0 && (flags == SLA_PCG_PERSISTENT || small);
  }
  if (flags == SLA_PCG_PERSISTENT && !persistent) return SLA_ERR_UNSUPPORTED;
  bool clustered = false;
  if (flags == SLA_PCG_CLUSTER || (flags == SLA_PCG_AUTO && persistent)) {
    cudaEvent_t ev;
    profiler().begin(0, 0, s, &ev);
    SLA_TRY((cluster_launch<T, PREC, WS>(A, n, x, r, dinv, st, s, &clustered)));
    profiler().end(0, s, ev);
    if (flags == SLA_PCG_CLUSTER && !clustered) return SLA_ERR_UNSUPPORTED;
  }

  if (clustered) {
    // the whole solve ran in the cluster kernel
  } else if (persistent) {
    int64_t nn = n;
    void *args[] = {&A, &nn, &x, &r, (void *)&dinv, &pA, &pB, &Ap, &st, &part0, &part1};
    cudaEvent_t ev;
    profiler().begin(0, 0, s, &ev);
    SLA_CUDA_TRY(cudaLaunchCooperativeKernel((const void *)cg_persistent_kernel<T, PREC, WS>,
                                             dim3(coop_grid), dim3(kPBlock), args, 0, s));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    profiler().end(0, s, ev);
  } else {
    KaLaunch<T, PREC, WS> ka;
    ka.init(n, r, dinv, pA, pB);
    const bool vec = aligned16(x, r, pA, pB, Ap) && (!PREC || aligned16(dinv));
    SLA_TRY(run_chunked(maxiter, 8, &st->done, s, [&](int64_t it) -> int {
      T *p_old = (it & 1) ? pB : pA;
      T *p_new = (it & 1) ? pA : pB;
      cudaEvent_t ev;
      SLA_TRY(ka.run(it, true, A, r, dinv, p_old, p_new, Ap, st, part0, s));
      profiler().begin(1, it, s, &ev);
      SLA_TRY((update_launch<T, PREC>(vec, it, n, x, r, p_new, p_old, Ap, dinv, st, part1, s)));
      profiler().end(1, s, ev);
      return SLA_OK;
    }));
    // pending x step of a last even iteration (its direction sits in pB)
    SLA_LAUNCH(cg_xflush_kernel<T>, grid_for(n), kBlock, 0, s, n, x, pB, st);
  }
  CgState out;
  SLA_CUDA_TRY(cudaMemcpyAsync(&out, st, sizeof(CgState), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  profiler().resolve();
  info->residual = sqrt(out.rr);
  info->reason = out.done;
  if (out.done == kTimeout) return SLA_ERR_TIMEOUT;
  info->iterations = out.iters_out;
  info->status = out.done == kConverged ? SLA_OK : SLA_NOT_CONVERGED;
  return info->status;
}

// ------------------------------------------------- allocation-free variant
// Scratch of sla_pcg_noalloc: one file-scope device array, present on every
// GPU that loads the library. In host code the symbol is only a handle, never
// a device address; the address is resolved per device with
// cudaGetSymbolAddress and passed to the kernels.
static __device__ __align__(256) unsigned char g_pcg_noalloc_scratch[SLA_PCG_NOALLOC_SCRATCH_BYTES];

// Device address of the scratch array on the current device. It is resolved
// on every call (cudaGetSymbolAddress is cheap next to a solve), so an
// address can never go stale, e.g. after a cudaDeviceReset reloads the module.
static int noalloc_scratch(void **out) {
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_pcg_noalloc_scratch);
  if (e != cudaSuccess || !p) {
    fprintf(stderr, "[sla_b200] cudaGetSymbolAddress(pcg scratch) failed: %s\n",
            cudaGetErrorString(e));
    return SLA_ERR_CUDA;
  }
  *out = p;
  return SLA_OK;
}

// Same kernels and launch shapes as pcg_impl; the convergence flag is polled
// with a plain stream-ordered copy (no pinned buffer, no events).
template <typename T, bool PREC, int WS>
static int pcg_noalloc_impl(const sla_sell_t *Ad, const T *dinv, const T *b, T *x, bool guess,
                            double atol, double rtol, int64_t maxiter, int flags, void *ws,
                            size_t ws_bytes, sla_solve_info_t *info, cudaStream_t s) {
  Sell<T> A = make_sell<T>(Ad);
  const int64_t n = A.n_slots;
  Carver c(ws, ws_bytes);
  T *r = c.take<T>(n), *pA = c.take<T>(n), *pB = c.take<T>(n), *Ap = c.take<T>(n);
  const int G = solver_grid();
  double *part0 = c.take<double>(4 * (size_t)G), *part1 = c.take<double>(4 * (size_t)G);
  CgState *st = c.take<CgState>(1);
  if (!c.ok) return SLA_ERR_UNSUPPORTED;
  CgState init{};
  init.maxiter = maxiter;
  SLA_CUDA_TRY(cudaMemcpyAsync(st, &init, sizeof(CgState), cudaMemcpyHostToDevice, s));
  if (guess) SLA_TRY(spmv_launch<T>(Ad, x, Ap, s));
  SLA_LAUNCH((cg_init_kernel<T, PREC>), grid_for(n), kBlock, 0, s, n, b, x, guess ? Ap : nullptr,
             dinv, r, pA, st, part0, atol, rtol);
  const DeviceInfo &dev = device_info();
  bool persistent = false;
  int coop_grid = 0;
  if (flags != SLA_PCG_STREAMED && dev.coop) {
    int per_sm = 0;
    SLA_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(
        &per_sm, cg_persistent_kernel<T, PREC, WS>, kPBlock, 0));
    int want = (int)((n + kPBlock - 1) / kPBlock);
    int cap = per_sm * dev.sm_count;
    coop_grid = want < cap ? want : cap;
    if (coop_grid < 1) coop_grid = 1;
    // the same rule as pcg_impl: AUTO keeps large systems on the streamed path
    bool small = n <= (int64_t)(1 << 20);
    persistent = per_sm > 0 && (flags == SLA_PCG_PERSISTENT || small);
  }
  if (flags == SLA_PCG_PERSISTENT && !persistent) return SLA_ERR_UNSUPPORTED;
  bool clustered = false;
  if (flags == SLA_PCG_CLUSTER || (flags == SLA_PCG_AUTO && persistent)) {
    SLA_TRY((cluster_launch<T, PREC, WS>(A, n, x, r, dinv, st, s, &clustered)));
    if (flags == SLA_PCG_CLUSTER && !clustered) return SLA_ERR_UNSUPPORTED;
  }
  if (clustered) {
    // the whole solve ran in the cluster kernel
  } else if (persistent) {
    int64_t nn = n;
    void *args[] = {&A, &nn, &x, &r, (void *)&dinv, &pA, &pB, &Ap, &st, &part0, &part1};
    SLA_CUDA_TRY(cudaLaunchCooperativeKernel((const void *)cg_persistent_kernel<T, PREC, WS>,
                                             dim3(coop_grid), dim3(kPBlock), args, 0, s));
    g_launches.fetch_add(1, std::memory_order_relaxed);
  } else {
    KaLaunch<T, PREC, WS> ka;
    ka.init(n, r, dinv, pA, pB);
    for (int64_t it = 0; it < maxiter;) {
      int64_t chunk = maxiter - it < 8 ? maxiter - it : 8;
      for (int64_t j = 0; j < chunk; ++j, ++it) {
        T *p_old = (it & 1) ? pB : pA;
        T *p_new = (it & 1) ? pA : pB;
        SLA_TRY(ka.run(it, false, A, r, dinv, p_old, p_new, Ap, st, part0, s));
        const bool vec = aligned16(x, r, pA, pB, Ap) && (!PREC || aligned16(dinv));
        SLA_TRY((update_launch<T, PREC>(vec, it, n, x, r, p_new, p_old, Ap, dinv, st, part1, s)));
      }
      int done = 0;
      SLA_CUDA_TRY(cudaMemcpyAsync(&done, &st->done, sizeof(int), cudaMemcpyDeviceToHost, s));
      SLA_CUDA_TRY(cudaStreamSynchronize(s));
      if (done) break;
    }
    SLA_LAUNCH(cg_xflush_kernel<T>, grid_for(n), kBlock, 0, s, n, x, pB, st);
  }
  CgState out;
  SLA_CUDA_TRY(cudaMemcpyAsync(&out, st, sizeof(CgState), cudaMemcpyDeviceToHost, s));
  SLA_CUDA_TRY(cudaStreamSynchronize(s));
  info->residual = sqrt(out.rr);
  info->reason = out.done;
  if (out.done == kTimeout) return SLA_ERR_TIMEOUT;
  info->iterations = out.iters_out;
  info->status = out.done == kConverged ? SLA_OK : SLA_NOT_CONVERGED;
  return info->status;
}

}  // namespace sla

using namespace sla;

extern "C" {

int sla_pcg_workspace(int dtype, int64_t n, size_t *bytes) {
  if (!bytes || n < 0 || (dtype != SLA_F32 && dtype != SLA_F64)) return SLA_ERR_INVALID;
  *bytes = cg_ws_bytes(dtype == SLA_F64 ? 8 : 4, n);
  return SLA_OK;
}

int sla_pcg(int dtype, const sla_sell_t *A, const void *dinv, const void *b, void *x,
            int x_is_guess, double atol, double rtol, int64_t maxiter, int flags, void *workspace,
            size_t workspace_bytes, sla_solve_info_t *info, sla_stream_t stream) {
  SLA_TRY(sell_check(A));
  if (!b || !x || !info || A->row_base) return SLA_ERR_INVALID;
  if (A->n_diags > 0 && A->n_cols > A->n_slots) return SLA_ERR_INVALID;  // square system
  if (A->n_slots <= 0 || A->n_slots >= INT32_MAX) return SLA_ERR_INVALID;
  if (flags < 0 || flags > 3) return SLA_ERR_INVALID;
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  size_t need = 0;
  SLA_TRY(sla_pcg_workspace(dtype, A->n_slots, &need));
  if (workspace_bytes < need || !workspace) return SLA_ERR_WORKSPACE;
  cudaStream_t s = (cudaStream_t)stream;
  bool g = x_is_guess != 0;
  const int wspec = width_spec(A);
  if (dtype == SLA_F64) {
    if (dinv)
      SLA_WS_DISPATCH(wspec, return pcg_impl<double, true, WS>(A, (const double *)dinv, (const double *)b, (double *)x, g, atol,
                                    rtol, maxiter, flags, workspace, workspace_bytes, info, s));
    SLA_WS_DISPATCH(wspec, return pcg_impl<double, false, WS>(A, nullptr, (const double *)b, (double *)x, g, atol, rtol,
                                   maxiter, flags, workspace, workspace_bytes, info, s));
  }
  if (dtype == SLA_F32) {
    if (dinv)
      SLA_WS_DISPATCH(wspec, return pcg_impl<float, true, WS>(A, (const float *)dinv, (const float *)b, (float *)x, g, atol,
                                   rtol, maxiter, flags, workspace, workspace_bytes, info, s));
    SLA_WS_DISPATCH(wspec, return pcg_impl<float, false, WS>(A, nullptr, (const float *)b, (float *)x, g, atol, rtol, maxiter,
                                  flags, workspace, workspace_bytes, info, s));
  }
  return SLA_ERR_INVALID;
}

int sla_pcg_noalloc(int dtype, const sla_sell_t *A, const void *dinv, const void *b, void *x,
                    int x_is_guess, double atol, double rtol, int64_t maxiter, int flags,
                    sla_solve_info_t *info, sla_stream_t stream) {
  SLA_TRY(sell_check(A));
  if (!b || !x || !info || A->row_base) return SLA_ERR_INVALID;
  if (A->n_diags > 0 && A->n_cols > A->n_slots) return SLA_ERR_INVALID;  // square system
  if (A->n_slots <= 0 || A->n_slots >= INT32_MAX) return SLA_ERR_INVALID;
  if (flags < 0 || flags > 3) return SLA_ERR_INVALID;
  if (dtype != SLA_F32 && dtype != SLA_F64) return SLA_ERR_INVALID;
  info->iterations = 0; info->residual = 0; info->status = 0; info->reason = 0;
  size_t need = cg_ws_bytes(dtype == SLA_F64 ? 8 : 4, A->n_slots);
  if (need > (size_t)SLA_PCG_NOALLOC_SCRATCH_BYTES) {
    fprintf(stderr,
            "[sla_b200] sla_pcg_noalloc: n=%lld needs %zu scratch bytes, above the fixed "
            "%u-byte device array; use sla_pcg with a caller workspace\n",
            (long long)A->n_slots, need, (unsigned)SLA_PCG_NOALLOC_SCRATCH_BYTES);
    return SLA_ERR_UNSUPPORTED;
  }
  void *ws = nullptr;
  SLA_TRY(noalloc_scratch(&ws));
  const size_t cap = SLA_PCG_NOALLOC_SCRATCH_BYTES;
  cudaStream_t s = (cudaStream_t)stream;
  bool g = x_is_guess != 0;
  const int wspec = width_spec(A);
  if (dtype == SLA_F64) {
    if (dinv)
      SLA_WS_DISPATCH(wspec, return pcg_noalloc_impl<double, true, WS>(A, (const double *)dinv, (const double *)b,
                                            (double *)x, g, atol, rtol, maxiter, flags, ws, cap,
                                            info, s));
    SLA_WS_DISPATCH(wspec, return pcg_noalloc_impl<double, false, WS>(A, nullptr, (const double *)b, (double *)x, g, atol,
                                           rtol, maxiter, flags, ws, cap, info, s));
  }
  if (dinv)
    SLA_WS_DISPATCH(wspec, return pcg_noalloc_impl<float, true, WS>(A, (const float *)dinv, (const float *)b, (float *)x, g,
                                         atol, rtol, maxiter, flags, ws, cap, info, s));
  SLA_WS_DISPATCH(wspec, return pcg_noalloc_impl<float, false, WS>(A, nullptr, (const float *)b, (float *)x, g, atol, rtol,
                                        maxiter, flags, ws, cap, info, s));
}

}  // extern "C"
